// B200 batched token sampler: logits [B, V] -> token ids [B].
//
// One thread-block cluster of S CTAs (512 threads each) samples one row;
// each CTA owns a contiguous slice of it and reads every byte of the slice
// exactly once from HBM:
//
//   loads     the small per-row inputs first (history length and words,
//             parameter words, the slice's unaligned fringe, bias entries),
//             staged in shared memory before the slice is requested: issued
//             behind the slice they would wait for most of the 19 MB stream
//             of all rows.  Then the slice, as 1-D bulk copies into shared
//             memory (64 KB per mbarrier; every wait is bounded in time).
//   setup     while the copies land: a skip bitmap of the slice's special ids
//             (history / bias ids, allowed-mask holes), a seen map for
//             seen-bit penalties, the row's parameters and Philox uniform,
//             and a hash table of the specials with occurrence counts.
//   pass A    raw maximum per vector as each chunk lands, specials masked out
//             by a taint mask; a slice of at most 152 KB keeps each vector's
//             raw maximum in registers (19 vectors per thread, thread t
//             owning vectors t, t + 512, ...).  The specials' final values
//             (bias, penalties, mask, temperature) come from the table and,
//             for seen ids, straight from the resident data.
//   threshold theta(cm) from the CTA's own maximum: below it no value can
//             carry weight or pass min_p for any row maximum m >= cm, so no
//             cluster exchange is needed before candidates are chosen.
//   push      vectors whose raw maximum reaches theta are rescanned; their
//             candidates go straight into the leader CTA's shared memory
//             (one reservation per warp and step); a top_k row whose vectors above theta are many
//             times K is first cut below the value bin holding the K-th
//             largest vector maximum, and one that still holds more than it
//             may push is cut at its K-th largest value; the CTA's maximum,
//             count, status and lowest id at its maximum go to every peer.
//             One cluster barrier per step.
//   tail      (leader) rank sort, value-bucket sort (one atomic pass of
//             bucket counts and masses up to 512 candidates) or key-bucket
//             sort of the candidates, then top_k / top_p / the inverse-CDF draw from
//             exact u64 prefix sums of the fixed-point weights.  Rows with
//             more than 2048 candidates run the general path instead:
//             histogram (count + mass) and compaction rounds over the
//             still-resident slices until every boundary is pinned.
//   epilogue  id, status, stop flag, in-graph state updates (history ring,
//             seen bit, RNG offset).  MODE 1 (a vocabulary shard) emits the
//             shard's candidate record instead, merged by tp_merge_kernel.
//
// Rows of at most 4096 ids take small_kernel (one CTA, no cluster).  The
// LM-head projection that produces the logits is in lmhead.cuh.
//
// Reference call sites this kernel serves: CudaGraphableSampler.sample in
// python/mstar_rs/models/orpheus.py:350 and qwen3_omni.py:518 (batched,
// in-graph), Sampler.sample in orpheus.py:517 / qwen3_omni.py:483 (eager).
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/mstar_sampler.h"
#include "spec.cuh"

namespace cg = cooperative_groups;

namespace mstar {

constexpr int NT = 512;             // threads per CTA
constexpr int NWARP = NT / 32;
constexpr int TAIL_CAP = 2048;      // candidates the fast tail resolves
constexpr int LCAP = TAIL_CAP;      // CTA-local candidate list (general path)
constexpr int GCAP = 512;           // candidates per locate round of the general path
constexpr int NBIN_LOG2 = 10;
constexpr int NBIN = 1 << NBIN_LOG2;  // histogram bins per general-path round
constexpr int NBK_LOG2 = 11;
constexpr int NBK = 1 << NBK_LOG2;   // buckets of the fast tail
constexpr int GBK_LOG2 = 9;
constexpr int GBK = 1 << GBK_LOG2;   // buckets of the general-path sort
constexpr int CHUNK_BYTES = 65536;  // bulk-copy granule (one mbarrier each)
constexpr int MAX_CHUNKS = 4;       // slice data <= 256 KB
constexpr int MAX_ROUNDS = 96;      // bound on general-path rounds
constexpr int BIAS_SMEM = 256;      // bias entries staged in shared memory
constexpr int NPARAM = 7;           // per-row sampling parameter words
constexpr int PRECUT_FACTOR = 2;   // pre-cut a top_k row when more than this many times K vectors pass (2, not 4: bucket B=128 102.5 -> 98.4 us)
constexpr int GCUT_MAX_K = TAIL_CAP * 3 / 4;  // cluster-wide top_k cut up to this K (the cut's spill must fit the tail)
constexpr int NVR = 19;             // vectors per thread whose maxima stay in registers (152 KB per CTA)
constexpr int HIST_BYTES = NBIN * 16;  // per histogram: counts + three 11-bit mass parts
constexpr int GEN_BYTES = 2 * HIST_BYTES + GCAP * 8;  // L1 | REF (aliased by the sort scratch) | sort input
static_assert(NBIN * 8 <= NBIN * 12, "64-bit mass prefixes fit over the part arrays");
static_assert(GCAP * 20 + GBK * 8 <= HIST_BYTES, "general sort scratch");
static_assert(GBK * 8 >= 256 * 8 && GCAP >= 256, "small general sort: weights over the bucket arrays");
static_assert((NT / 32) * 256 * 4 <= HIST_BYTES && (NT / 32) * 256 <= LCAP * 2, "general-path warp lists");
static_assert(GBK <= NT && NBIN % NT == 0 && NBK % NT == 0 && TAIL_CAP % NT == 0, "per-thread splits");
constexpr int WORK_BYTES_MIN = GEN_BYTES;
constexpr int LEAN_SCRATCH = 112 * 1024;  // fast-tail scratch (the leader's data region)
static_assert(TAIL_CAP * 44 + NBK * 12 <= LEAN_SCRATCH, "fast tail scratch");
static_assert(NBK % NT == 0, "tail bucket scan");
static_assert(NBK >= 2 * 256 && NBK >= NT, "value-bucket tail: counts and starts over the bucket counts, weights over the masses");
static_assert(NT == 512, "the rank sort splits 512 threads into 64 / 128 / 256 slots");
// Bound on one wait for a bulk copy: 2 ms of %globaltimer (a copy of at
// most 64 KB lands within microseconds), with an iteration cap behind it.
constexpr uint64_t kWaitNs = 2000000ull;
constexpr unsigned kWaitIters = 1u << 26;

struct __align__(8) Cand {
  float x;
  uint32_t gid;
};

// Launch plan computed on the host (see plan_launch).
struct Plan {
  int32_t S;
  int32_t es;
  int64_t slice;       // elements per CTA slice
  int32_t data_bytes;  // slice data (>= LEAN_SCRATCH: reused by the fast tail)
  int32_t map_bytes;   // skip bitmap (one bit per resident position)
  int32_t seen_map;    // 1: a seen map of the same size follows the skip bitmap
  int32_t ht_cap;      // hash table slots (power of two)
  int32_t spec_cap;    // special list entries
  int32_t off_work, off_spec, off_lcand, off_bias;
  int32_t smem_bytes;
  int32_t mode;        // 0 = step, 1 = TP local
  int32_t tp_cap, rec_words;
  float *xdump;        // TP local, two rounds: shard values [B, V] of rows without a usable top_k
};

enum : int { OP_DONE = 0, OP_HIST = 1, OP_COMPACT = 2 };
enum : int { TGT_L1 = 0, TGT_REF = 1 };

struct Cmd {
  int op, target;
  uint64_t lo, hi;
  int shift, nbins;
};

enum : int {
  ST_START = 0,
  ST_AFTER_L1,
  ST_AFTER_PREFIX,
  ST_LOC_BIN,
  ST_LOC_AFTER_REF,
  ST_LOC_AFTER_COMPACT,
  ST_FINISH
};
enum : int { Q_COUNT = 0, Q_LASTLT = 1, Q_POINT = 2 };

struct Planner {
  int state;
  int stage;  // 0 = A boundary, 1 = top-p boundary, 2 = draw
  int qkind;
  int level;  // 0 = L1 arrays, 1 = REF arrays
  uint64_t lo, hi;
  int shift, nbins;
  uint64_t base_c, base_m;
  uint64_t l1lo, l1hi;
  int l1shift, l1nbins;
  uint64_t tcount, tpoint;
  double thr;
  uint64_t cbase_c, cbase_m;  // stats before the compacted bin
  uint64_t N, Wv, WA, WK, ckA, ckK;
};

struct Result {
  float m, theta;
  uint64_t WK, ckK;
  uint32_t token;
  uint32_t status;
  int greedy, empty;
};

struct Row {
  const void *rowp;
  int64_t V, gbase;  // gbase = vocab_offset
  float T, invT, Mp, lnMp, P;
  float R, F, Pp;    // repetition / frequency / presence penalties
  int K;             // 0 = off
  bool greedy, topk, minp, topp;
};

struct CtaSh {
  uint64_t mbar[MAX_CHUNKS];
  uint32_t red_u32[NWARP];
  float red_f[NWARP];
  uint64_t red_u64[NWARP];
  uint64_t red_u64b[NWARP];
  float maxes[16];    // per-CTA maxima, pushed by every CTA of the cluster
  uint32_t gstat[16];  // per-CTA status bits, pushed
  uint32_t gmin[16];   // per-CTA lowest id at the max (greedy / top-1), pushed
  uint32_t nloc;       // CTA-local candidate count
  uint32_t scanned;    // vectors a full candidate scan covered before it stopped (0: no full scan)
  uint32_t cmax;       // okey of the CTA max (transformed)
  uint32_t best;       // lowest id at the max (greedy / top-1)
  uint32_t status;     // status bits of this CTA
  uint64_t kmin, kmax;  // tail: key range
  uint32_t npass;       // tail: candidates passing the value-A predicate
  uint32_t cnt_k;       // tail: ranks kept by top_p
  float u;              // the row's uniform draw
  uint32_t n_spec;
  uint32_t ht_fail;
  float theta;
  float m;
  int fast;
  uint32_t ncand;
  uint32_t goff[16], gcnt[16];
  uint32_t min_all;
  int nemit;
  int kcut_bin;         // candidates: value bin of this CTA's K-th largest (top_k cut)
  uint32_t vcount;      // candidates: untainted vectors reaching theta (pre-cut)
  Row row;
  int tp_ovf;
  int pseudo;           // TP two rounds: the row's top_k is the record capacity
  int dumpx;            // TP two rounds: the shard values go to the value buffer
  int bcast_i;
  uint64_t bcast_u64;
  uint32_t pw[NPARAM];  // the row's parameter words, staged for row_init
  uint64_t rng[2];      // the row's uniform (bits) or Philox seed, and offset
  Cmd cmd;
  Planner pl;
  Result res;
};

// ---------------------------------------------------------------- helpers

__device__ __forceinline__ uint64_t u64min(uint64_t a, uint64_t b) { return a < b ? a : b; }
__device__ __forceinline__ uint64_t u64max(uint64_t a, uint64_t b) { return a > b ? a : b; }

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// First of `cnt` consecutive slots in a shared list for each lane of a full
// warp (all 32 lanes call it together): one atomic per warp.
__device__ __forceinline__ uint32_t warp_reserve(uint32_t *counter, uint32_t cnt) {
  const int lane = threadIdx.x & 31;
  uint32_t inc = cnt;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(~0u, inc, o);
    if (lane >= o) inc += t;
  }
  const uint32_t tot = __shfl_sync(~0u, inc, 31);
  uint32_t base = 0;
  if (lane == 31 && tot) base = atomicAdd(counter, tot);
  return __shfl_sync(~0u, base, 31) + inc - cnt;
}

// 64-bit sums in shared (or cluster shared) memory kept as two 32-bit words
// lo[i], hi[i]: 32-bit atomics are native, 64-bit atomic adds are
// compare-and-swap loops that serialise badly under contention.
__device__ __forceinline__ void add_u64_split(uint32_t *lo, uint32_t *hi, uint64_t v) {
  const uint32_t vl = (uint32_t)v;
  uint32_t vh = (uint32_t)(v >> 32);
  if (vl) {
    const uint32_t old = atomicAdd(lo, vl);
    vh += (old + vl < old) ? 1u : 0u;  // carry out of the low word
  }
  if (vh) atomicAdd(hi, vh);
}
__device__ __forceinline__ uint64_t get_u64_split(const uint32_t *lo, const uint32_t *hi) {
  return ((uint64_t)*hi << 32) | *lo;
}

// Split cluster barrier: a CTA may touch a peer's shared memory only once
// the peer is known to run, i.e. after a wait matching every CTA's arrive.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on phase `parity` (kWaitNs); false if the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (unsigned i = 0; i < kWaitIters; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    const uint64_t t = global_ns();
    if (i == 0) t0 = t;
    else if (t - t0 > kWaitNs) return false;
  }
  return false;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static constexpr int VEC = 4;
  // running-max accumulator of the first pass
  using Acc = float;
  static __device__ __forceinline__ Acc acc_init() { return -INFINITY; }
  static __device__ __forceinline__ Acc vred(const uint4 &v) {
    return fmaxf(fmaxf(__uint_as_float(v.x), __uint_as_float(v.y)), fmaxf(__uint_as_float(v.z), __uint_as_float(v.w)));
  }
  static __device__ __forceinline__ Acc acc_max(Acc a, Acc b) { return fmaxf(a, b); }
  static __device__ __forceinline__ float acc_f(Acc a) { return a; }
  static __device__ __forceinline__ float get(const uint4 &v, int j) {
    const uint32_t w = j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
    return __uint_as_float(w);
  }
  static __device__ __forceinline__ void set_bits(uint4 &v, int j, uint32_t bits) {
    if (j == 0) v.x = bits;
    else if (j == 1) v.y = bits;
    else if (j == 2) v.z = bits;
    else v.w = bits;
  }
  static __device__ __forceinline__ float vmax(const uint4 &v) {
    return fmaxf(fmaxf(__uint_as_float(v.x), __uint_as_float(v.y)),
                 fmaxf(__uint_as_float(v.z), __uint_as_float(v.w)));
  }
  static __device__ __forceinline__ float load(const void *row, int64_t i) {
    return static_cast<const float *>(row)[i];
  }
  static __device__ __forceinline__ uint32_t load_bits(const void *row, int64_t i) {
    return static_cast<const uint32_t *>(row)[i];
  }
  static __device__ __forceinline__ uint32_t neg_inf() { return 0xFF800000u; }
  static __device__ __forceinline__ uint32_t nan_bits() { return 0x7FC00000u; }
  static __device__ __forceinline__ uint32_t bits_of(const uint8_t *map, int k) {
    return (map[k >> 1] >> ((k & 1) * 4)) & 0xFu;
  }
  // lanes whose bit is set become -inf
  static __device__ __forceinline__ uint4 mask_out(uint4 v, uint32_t b) {
    v.x = (b & 1u) ? 0xFF800000u : v.x;
    v.y = (b & 2u) ? 0xFF800000u : v.y;
    v.z = (b & 4u) ? 0xFF800000u : v.z;
    v.w = (b & 8u) ? 0xFF800000u : v.w;
    return v;
  }
  static __device__ __forceinline__ float smem_elem(const uint8_t *data, int64_t pos) {
    return reinterpret_cast<const float *>(data)[pos];
  }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int VEC = 8;
  // running-max accumulator of the first pass: a bf16 pair (max of the
  // even and of the odd lanes), reduced to one float only when read
  using Acc = uint32_t;
  static __device__ __forceinline__ Acc acc_init() { return 0xFF80FF80u; }
  static __device__ __forceinline__ Acc hmax_bits(uint32_t a, uint32_t b) {
    const __nv_bfloat162 r = __hmax2(*reinterpret_cast<const __nv_bfloat162 *>(&a),
                                     *reinterpret_cast<const __nv_bfloat162 *>(&b));
    return *reinterpret_cast<const uint32_t *>(&r);
  }
  static __device__ __forceinline__ Acc vred(const uint4 &v) {
    return hmax_bits(hmax_bits(v.x, v.y), hmax_bits(v.z, v.w));
  }
  static __device__ __forceinline__ Acc acc_max(Acc a, Acc b) { return hmax_bits(a, b); }
  static __device__ __forceinline__ float acc_f(Acc a) {
    return fmaxf(__uint_as_float(a << 16), __uint_as_float(a & 0xFFFF0000u));
  }
  static __device__ __forceinline__ float get(const uint4 &v, int j) {
    const uint32_t w = (j >> 1) == 0 ? v.x : (j >> 1) == 1 ? v.y : (j >> 1) == 2 ? v.z : v.w;
    return __uint_as_float((j & 1) ? (w & 0xFFFF0000u) : (w << 16));
  }
  static __device__ __forceinline__ void set_bits(uint4 &v, int j, uint32_t bits) {
    const uint32_t hi = (j & 1) ? 0x0000FFFFu : 0xFFFF0000u;  // half to keep
    const uint32_t put = (j & 1) ? (bits << 16) : (bits & 0xFFFFu);
    const int w = j >> 1;
    if (w == 0) v.x = (v.x & hi) | put;
    else if (w == 1) v.y = (v.y & hi) | put;
    else if (w == 2) v.z = (v.z & hi) | put;
    else v.w = (v.w & hi) | put;
  }
  static __device__ __forceinline__ float vmax(const uint4 &v) {
    __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162 *>(&v.x);
    __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162 *>(&v.y);
    __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162 *>(&v.z);
    __nv_bfloat162 d = *reinterpret_cast<const __nv_bfloat162 *>(&v.w);
    a = __hmax2(__hmax2(a, b), __hmax2(c, d));
    return fmaxf(__low2float(a), __high2float(a));
  }
  static __device__ __forceinline__ float load(const void *row, int64_t i) {
    const uint16_t h = static_cast<const uint16_t *>(row)[i];
    return __uint_as_float((uint32_t)h << 16);
  }
  static __device__ __forceinline__ uint32_t load_bits(const void *row, int64_t i) {
    return static_cast<const uint16_t *>(row)[i];
  }
  static __device__ __forceinline__ uint32_t neg_inf() { return 0xFF80u; }
  static __device__ __forceinline__ uint32_t nan_bits() { return 0x7FC0u; }
  static __device__ __forceinline__ uint32_t bits_of(const uint8_t *map, int k) { return map[k]; }
  static __device__ __forceinline__ uint32_t mask2(uint32_t w, uint32_t b2) {
    const uint32_t m = ((b2 & 1u) ? 0x0000FFFFu : 0u) | ((b2 & 2u) ? 0xFFFF0000u : 0u);
    return (w & ~m) | (0xFF80FF80u & m);
  }
  // lanes whose bit is set become -inf
  static __device__ __forceinline__ uint4 mask_out(uint4 v, uint32_t b) {
    v.x = mask2(v.x, b);
    v.y = mask2(v.y, b >> 2);
    v.z = mask2(v.z, b >> 4);
    v.w = mask2(v.w, b >> 6);
    return v;
  }
  static __device__ __forceinline__ float smem_elem(const uint8_t *data, int64_t pos) {
    return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(data)[pos] << 16);
  }
};

// ------------------------------------------------------- block reductions

__device__ __forceinline__ float block_max_f32(float v, CtaSh &sh) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(~0u, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.red_f[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = sh.red_f[0];
  for (int i = 1; i < NWARP; ++i) r = fmaxf(r, sh.red_f[i]);
  return r;
}

__device__ __forceinline__ uint32_t block_min_u32(uint32_t v, CtaSh &sh) {
  for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(~0u, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.red_u32[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = sh.red_u32[0];
  for (int i = 1; i < NWARP; ++i) r = min(r, sh.red_u32[i]);
  return r;
}

__device__ __forceinline__ void block_minmax_u64(uint64_t &mn, uint64_t &mx, CtaSh &sh) {
  for (int o = 16; o; o >>= 1) {
    mn = u64min(mn, (uint64_t)__shfl_xor_sync(~0u, (unsigned long long)mn, o));
    mx = u64max(mx, (uint64_t)__shfl_xor_sync(~0u, (unsigned long long)mx, o));
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    sh.red_u64[threadIdx.x >> 5] = mn;
    sh.red_u64b[threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  mn = sh.red_u64[0];
  mx = sh.red_u64b[0];
  for (int i = 1; i < NWARP; ++i) {
    mn = u64min(mn, sh.red_u64[i]);
    mx = u64max(mx, sh.red_u64b[i]);
  }
}

// Exclusive block scan (one value per thread); returns the prefix and the total.
__device__ __forceinline__ uint64_t block_exscan_u64(uint64_t v, uint64_t &total, CtaSh &sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint64_t inc = v;
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t t = __shfl_up_sync(~0u, (unsigned long long)inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) sh.red_u64[wid] = inc;
  __syncthreads();
  uint64_t off = 0, tot = 0;
  for (int i = 0; i < NWARP; ++i) {
    const uint64_t s = sh.red_u64[i];
    if (i < wid) off += s;
    tot += s;
  }
  total = tot;
  return off + inc - v;
}

// Two exclusive block scans at once (count and mass).
__device__ __forceinline__ void block_exscan2_u64(uint64_t a, uint64_t b, uint64_t &pa, uint64_t &pb, uint64_t &ta,
                                                  uint64_t &tb, CtaSh &sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint64_t ia = a, ib = b;
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t sa = __shfl_up_sync(~0u, (unsigned long long)ia, o);
    const uint64_t sb = __shfl_up_sync(~0u, (unsigned long long)ib, o);
    if (lane >= o) {
      ia += sa;
      ib += sb;
    }
  }
  __syncthreads();
  if (lane == 31) {
    sh.red_u64[wid] = ia;
    sh.red_u64b[wid] = ib;
  }
  __syncthreads();
  uint64_t oa = 0, ob = 0, sa_ = 0, sb_ = 0;
  for (int i = 0; i < NWARP; ++i) {
    const uint64_t x = sh.red_u64[i], y = sh.red_u64b[i];
    if (i < wid) {
      oa += x;
      ob += y;
    }
    sa_ += x;
    sb_ += y;
  }
  pa = oa + ia - a;
  pb = ob + ib - b;
  ta = sa_;
  tb = sb_;
}

// ---------------------------------------------------------- row context




// The row's sampling parameters as raw 32-bit words, in the order
// temperature, top_k, min_p, top_p, repetition, frequency, presence
// (defaults for absent arrays); word j is loaded by one thread.
__device__ __forceinline__ uint32_t param_word(const mstar_sampler_params_t &p, int j, int slot) {
  switch (j) {
    case 0: return p.temperature ? __float_as_uint(p.temperature[slot]) : __float_as_uint(1.0f);
    case 1: return p.top_k ? (uint32_t)p.top_k[slot] : 0u;
    case 2: return p.min_p ? __float_as_uint(p.min_p[slot]) : 0u;
    case 3: return p.top_p ? __float_as_uint(p.top_p[slot]) : __float_as_uint(1.0f);
    case 4: return p.rep_pen ? __float_as_uint(p.rep_pen[slot]) : __float_as_uint(1.0f);
    case 5: return p.freq_pen ? __float_as_uint(p.freq_pen[slot]) : 0u;
    default: return p.pres_pen ? __float_as_uint(p.pres_pen[slot]) : 0u;
  }
}

__device__ __forceinline__ void row_init(Row &r, const uint32_t *w, const mstar_sampler_params_t &p, int row,
                                         int64_t V) {
  r.V = V;
  r.gbase = p.vocab_offset;
  const int es = p.dtype == MSTAR_DTYPE_BF16 ? 2 : 4;
  r.rowp = static_cast<const uint8_t *>(p.logits) + (int64_t)row * p.ld * es;
  r.T = __uint_as_float(w[0]);
  r.greedy = !(r.T >= 1e-5f);
  r.invT = r.greedy ? 1.0f : __fdiv_rn(1.0f, r.T);
  const int K = (int)w[1];
  r.topk = K > 0 && (int64_t)K < r.V;
  r.K = r.topk ? K : 0;
  const float Mp = __uint_as_float(w[2]);
  r.minp = Mp > 0.0f;
  r.Mp = fminf(Mp, 1.0f);
  r.lnMp = r.minp ? logf(r.Mp) : 0.0f;
  r.P = __uint_as_float(w[3]);
  r.topp = r.P < 1.0f;
  r.R = __uint_as_float(w[4]);
  r.F = __uint_as_float(w[5]);
  r.Pp = __uint_as_float(w[6]);
}

__device__ __forceinline__ void row_init(Row &r, const mstar_sampler_params_t &p, int row, int slot, int64_t V) {
  uint32_t w[NPARAM];
#pragma unroll
  for (int j = 0; j < NPARAM; ++j) w[j] = param_word(p, j, slot);
  row_init(r, w, p, row, V);
}

// value-A predicate of x given the row max m (positive weight and min_p).
__device__ __forceinline__ bool pred_A(const Row &r, float x, float m) {
  const float e = spec_e(x, m);
  if (spec_w_from_e(e) == 0) return false;
  return !r.minp || e >= r.Mp;
}

// Same predicate, also returning the fixed-point weight (0 when false).
__device__ __forceinline__ uint64_t weight_A(const Row &r, float x, float m) {
  const float e = spec_e(x, m);
  const uint64_t w = spec_w_from_e(e);
  if (w == 0 || (r.minp && !(e >= r.Mp))) return 0;
  return w;
}

__device__ __forceinline__ float prev_float(float t) {
  if (t != t || t == -INFINITY) return t;
  if (t == 0.0f) return -1.4e-45f;
  const int b = __float_as_int(t);
  return __int_as_float(t > 0.0f ? b - 1 : b + 1);
}

// Conservative value threshold: every x below it fails the value-A
// predicate.  Guesses of the boundary, each checked with the spec's own
// exponential at prev_float(theta) (the predicate is monotone in x); lanes
// 0-2 try the positive-weight bound, lanes 3-5 the min_p bound.  Called by
// one full warp; every lane returns the same value.
__device__ float choose_theta(const Row &r, float m) {
  if (r.greedy || r.K == 1) return m;
  const int lane = threadIdx.x & 31;
  float t = -INFINITY;
  bool ok = false;
  if (lane < 3) {
    const float off = lane == 0 ? -23.25f : lane == 1 ? -25.0f : -32.0f;
    t = __fadd_rn(m, off);
    ok = spec_w_from_e(spec_e(prev_float(t), m)) == 0;
  } else if (lane < 6 && r.minp) {
    const float off = lane == 3 ? -0.002f : lane == 4 ? -0.1f : -1.0f;
    t = __fadd_rn(m, __fadd_rn(r.lnMp, off));
    ok = !(spec_e(prev_float(t), m) >= r.Mp);
  }
  const unsigned bal = __ballot_sync(~0u, ok);
  const unsigned bw = bal & 7u, bm = (bal >> 3) & 7u;
  const float tw = bw ? __shfl_sync(~0u, t, __ffs(bw) - 1) : -INFINITY;
  const float tm = bm ? __shfl_sync(~0u, t, __ffs(bm) + 2) : -INFINITY;
  return fmaxf(tw, tm);
}

__device__ __forceinline__ uint64_t ckey(uint32_t km, float x, uint32_t gid) {
  return ((uint64_t)(km - okey(x)) << 32) | gid;
}

// Resident slice view used by the scans: data vectors plus the skip bitmap
// (positions outside the slice, disallowed by the mask, or special: their
// final value lives in the special list); skipped lanes read as -inf.
struct Slice {
  const uint4 *data;
  const uint8_t *skip;
  int nvec;
  int64_t pos0_gid;
  const uint32_t *seen;  // seen map (seen-bit mode) or NULL
  int map_words;         // words of the skip and seen maps
  const uint8_t *rowp;   // the row in global memory
  int64_t c0al;          // row position of data position 0
};

// Final value of a seen-mask special at data position pos (count 1; no
// bias: bias ids are in the materialized list), from the resident data or,
// with rowp, from global memory.  Same operations as the list's finalize.
template <typename T>
__device__ __forceinline__ float seen_x(const Slice &sl, int pos, const Row &r, bool from_global) {
  float v = from_global ? Elem<T>::load(sl.rowp, sl.c0al + pos)
                        : Elem<T>::smem_elem(reinterpret_cast<const uint8_t *>(sl.data), pos);
  v = (v > 0.0f) ? __fdiv_rn(v, r.R) : __fmul_rn(v, r.R);
  v = __fsub_rn(v, __fmul_rn(r.F, 1.0f));
  v = __fsub_rn(v, r.Pp);
  return v != v ? v : (r.greedy ? v : __fmul_rn(v, r.invT));
}

// The seen-mask specials of the slice as a list that is never materialized:
// every set bit of the seen map (a seen, allowed id that is not a bias id)
// is visited and its final value computed on the spot, so the number of
// seen ids a row may carry is not bounded by a shared-memory list.
// fn(c, valid) is called by all 32 lanes of each participating warp (the
// threads t0 = 0 .. stride-1 of the group, whole warps); no barrier.
template <typename T, typename F>
__device__ __forceinline__ void for_each_seen(const Slice &sl, const Row &r, bool from_global, int t0, int stride,
                                              F &&fn) {
  if (!sl.seen) return;
  const int lane = threadIdx.x & 31;
  for (int w0 = t0 & ~31; w0 < sl.map_words; w0 += stride) {  // warp-uniform
    const int wi = w0 + lane;
    uint32_t bits = wi < sl.map_words ? sl.seen[wi] : 0u;
    while (__any_sync(~0u, bits != 0u)) {
      const bool valid = bits != 0u;
      Cand c{-INFINITY, 0u};
      if (valid) {
        const int pos = wi * 32 + __ffs(bits) - 1;
        bits &= bits - 1u;
        c.x = seen_x<T>(sl, pos, r, from_global);
        c.gid = (uint32_t)(sl.pos0_gid + pos);
      }
      fn(c, valid);
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 load_masked(const Slice &sl, int k) {
  const uint4 v = sl.data[k];
  const uint32_t b = Elem<T>::bits_of(sl.skip, k);
  return b ? Elem<T>::mask_out(v, b) : v;
}

// Iterate the value-A elements this CTA holds whose order key lies in
// [lo, hi] (resident vectors and the special list), calling
// fn(x, gid, w, valid) with all 32 lanes of each warp, valid = the lane holds
// such an element (w its weight, > 0).  Each warp alternates a compact scan,
// which lists the vectors that may hold an element in range (their max
// reaches the range; unless DENSE, also one element inside its value
// bounds) in its own list (wq, QW entries), and an evaluation of the listed
// vectors 32 at a time, each lane evaluating its vector's elements together
// without branches so their exponentials overlap.  Keeping the two loops
// apart keeps the scan loop small.  Block-wide, warp-synchronous; no barrier.
constexpr int QW = 256;  // per-warp list entries (vector indices)
template <typename T, bool DENSE, typename F>
__device__ __forceinline__ void for_each_value(const Slice &sl, const Cand *spec, int nspec, const Row &r, float m,
                                               float theta, uint64_t lo, uint64_t hi, int *wq, F &&fn) {
  constexpr int VEC = Elem<T>::VEC;
  constexpr int SU = 4;  // vectors per lane per scan trip (independent loads in flight)
  const int lane = threadIdx.x & 31;
  const uint32_t km = okey(m);
  const uint32_t dhi = (uint32_t)(hi >> 32);
  const float xlo = dhi >= km ? -INFINITY : okey_inv(km - dhi);  // keys <= hi have x >= xlo
  const float tq = fmaxf(theta, xlo);
  const uint32_t dlo = (uint32_t)(lo >> 32);
  const float xhi = dlo == 0 ? INFINITY : okey_inv(km - dlo);  // keys >= lo have x <= xhi
  // the whole A range (keys 0 .. (km - okey(theta)) << 32 | ~0): x >= theta says it all
  const bool whole = lo == 0 && (hi >> 32) == (uint64_t)(km - okey(theta)) && (uint32_t)hi == 0xFFFFFFFFu;
  auto in_range = [&](float x, uint32_t gid) {
    if (!(x >= tq && x <= xhi)) return false;
    if (whole) return true;
    const uint64_t ck = ckey(km, x, gid);
    return ck >= lo && ck <= hi;
  };
  int kb = threadIdx.x & ~31;
  while (kb < sl.nvec) {  // warp-uniform
    int qn = 0;
    for (; kb < sl.nvec && qn <= QW - SU * 32; kb += SU * NT) {
      bool pv[SU];
#pragma unroll
      for (int u = 0; u < SU; ++u) {
        const int k = kb + u * NT + lane;
        pv[u] = false;
        if (k < sl.nvec) {
          const uint4 v = load_masked<T>(sl, k);
          if (DENSE) {
            const float vm = Elem<T>::vmax(v);
            pv[u] = (r.greedy ? vm : __fmul_rn(vm, r.invT)) >= tq;
          } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
              const float raw = Elem<T>::get(v, j);
              const float x = r.greedy ? raw : __fmul_rn(raw, r.invT);
              pv[u] |= x >= tq && x <= xhi;
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < SU; ++u) {
        const unsigned bal = __ballot_sync(~0u, pv[u]);
        if (pv[u]) wq[qn + __popc(bal & ((1u << lane) - 1u))] = kb + u * NT + lane;
        qn += __popc(bal);
      }
    }
    __syncwarp();
    for (int i = 0; i < qn; i += 32) {
      const bool have = i + lane < qn;
      const int k = have ? wq[i + lane] : 0;
      const uint4 v = have ? load_masked<T>(sl, k) : make_uint4(0, 0, 0, 0);
      const uint32_t gid0 = (uint32_t)(sl.pos0_gid + (int64_t)k * VEC);
      float x[VEC];
      uint64_t w[VEC];
      bool in[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float raw = Elem<T>::get(v, j);
        x[j] = r.greedy ? raw : __fmul_rn(raw, r.invT);
        in[j] = have && in_range(x[j], gid0 + (uint32_t)j);
        w[j] = weight_A(r, x[j], m);
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) fn(x[j], gid0 + (uint32_t)j, w[j], in[j] && w[j] != 0);
    }
    __syncwarp();
  }
  for (int ib = threadIdx.x & ~31; ib < nspec; ib += NT) {
    const int i = ib + lane;
    const Cand c = i < nspec ? spec[i] : Cand{-INFINITY, 0u};
    const bool in = i < nspec && in_range(c.x, c.gid);
    const uint64_t w = weight_A(r, c.x, m);
    fn(c.x, c.gid, w, in && w != 0);
  }
  for_each_seen<T>(sl, r, false, threadIdx.x, NT, [&](const Cand &c, bool valid) {
    const bool in = valid && in_range(c.x, c.gid);
    const uint64_t w = weight_A(r, c.x, m);
    fn(c.x, c.gid, w, in && w != 0);
  });
}

// ------------------------------------------------------------- fast tail

// --------------------------------------------------- general-path sort

struct SortScratch {
  Cand *in;  // [GCAP]
  Cand *mid;
  uint32_t *tmp;
  uint64_t *S;
  uint32_t *bcnt, *boff;
};

// Sort in[0..n) by (x desc, gid asc) in place; S[j] = inclusive prefix of
// the weights.  Block-wide.
__device__ void tail_sort_scan(Cand *in, int n, float m, const SortScratch &s, CtaSh &sh) {
  const uint32_t km = okey(m);
  uint64_t kmin = ~0ull, kmax = 0;
  for (int i = threadIdx.x; i < n; i += NT) {
    const uint64_t k = ckey(km, in[i].x, in[i].gid);
    kmin = u64min(kmin, k);
    kmax = u64max(kmax, k);
  }
  block_minmax_u64(kmin, kmax, sh);
  const uint64_t span = n > 0 ? kmax - kmin : 0;
  const int bits = span ? 64 - __clzll((long long)span) : 0;
  const int shift = bits > GBK_LOG2 ? bits - GBK_LOG2 : 0;  // (key - kmin) >> shift < GBK
  for (int b = threadIdx.x; b < GBK; b += NT) s.bcnt[b] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += NT) {
    const uint32_t b = (uint32_t)((ckey(km, in[i].x, in[i].gid) - kmin) >> shift);
    const uint32_t pos = atomicAdd(&s.bcnt[b], 1u);
    s.tmp[i] = (b << 16) | pos;
  }
  __syncthreads();
  {  // exclusive scan of the bucket counts (GBK <= NT: one bucket per thread)
    const uint32_t c = threadIdx.x < GBK ? s.bcnt[threadIdx.x] : 0u;
    uint64_t tot;
    const uint32_t off = (uint32_t)block_exscan_u64(c, tot, sh);
    if (threadIdx.x < GBK) s.boff[threadIdx.x] = off;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += NT) {
    const uint32_t t = s.tmp[i];
    s.mid[s.boff[t >> 16] + (t & 0xFFFFu)] = in[i];
  }
  __syncthreads();
  for (int q = threadIdx.x; q < n; q += NT) {
    const Cand c = s.mid[q];
    const uint64_t key = ckey(km, c.x, c.gid);
    const uint32_t b = (uint32_t)((key - kmin) >> shift);
    const uint32_t st = s.boff[b], cn = s.bcnt[b];
    uint32_t rank = 0;
    for (uint32_t j = st; j < st + cn; ++j) {
      const Cand o = s.mid[j];
      rank += ckey(km, o.x, o.gid) < key;
    }
    in[st + rank] = c;
  }
  __syncthreads();
  const int seg = (n + NT - 1) / NT;
  const int a = min(n, (int)threadIdx.x * seg), bnd = min(n, a + seg);
  uint64_t loc = 0;
  for (int j = a; j < bnd; ++j) {
    const uint64_t w = spec_w_from_e(spec_e(in[j].x, m));
    loc += w;
    s.S[j] = w;
  }
  uint64_t tot;
  uint64_t run = block_exscan_u64(loc, tot, sh);
  for (int j = a; j < bnd; ++j) {
    run += s.S[j];
    s.S[j] = run;
  }
  __syncthreads();
}

// tail_sort_scan for n <= 256 by pairwise counting (G = NT / slots
// threads per element, as in tail_rank_sort): every element's rank and the
// sum of the weights of the smaller keys in one pass.  Block-wide; ends with
// a barrier.
__device__ void tail_sort_scan_small(Cand *in, int n, float m, const SortScratch &s) {
  const uint32_t km = okey(m);
  const int t = threadIdx.x;
  const int G = n <= 64 ? NT / 64 : n <= 128 ? NT / 128 : NT / 256;
  const int e = t / G, part = t % G;
  uint64_t *K = reinterpret_cast<uint64_t *>(s.mid);   // [GCAP] keys
  uint64_t *W = reinterpret_cast<uint64_t *>(s.bcnt);  // [GBK] weights (bcnt and boff together)
  Cand c{0.0f, 0u};
  uint64_t key = ~0ull, w = 0;
  if (e < n) {
    c = in[e];
    key = ckey(km, c.x, c.gid);
    w = spec_w_from_e(spec_e(c.x, m));
    if (part == 0) {
      K[e] = key;
      W[e] = w;
    }
  }
  __syncthreads();  // keys and weights in; every element read from `in`
  uint32_t rk = 0;
  uint64_t before = 0;
#pragma unroll 4
  for (int j = part; j < n; j += G) {  // branch-free: loads of later j overlap
    const bool lt = K[j] < key;
    const uint64_t wj = W[j];
    rk += lt ? 1u : 0u;
    before += lt ? wj : 0ull;
  }
  for (int o = G >> 1; o; o >>= 1) {
    rk += __shfl_xor_sync(~0u, rk, o);
    before += (uint64_t)__shfl_xor_sync(~0u, (unsigned long long)before, o);
  }
  if (part == 0 && e < n) {
    in[rk] = c;
    s.S[rk] = before + w;
  }
  __syncthreads();
}

__device__ __forceinline__ uint64_t S_excl(const uint64_t *S, int j) { return j ? S[j - 1] : 0; }

// ------------------------------------------------------- kernel sections

struct Layout {
  uint8_t *data;
  uint8_t *skip;
  uint32_t *seen;  // seen-bit mode: seen, allowed, non-bias positions (or NULL)
  int2 *ht;    // {pos, count | HT_MASKED}
  int *queue;  // [NBIN] counts of the top_k cut's histogram
  Cand *spec;
  Cand *lcand;  // leader: candidates pushed by every CTA; general path: CTA-local list
  int32_t *bias_id;
  float *bias_val;
  uint8_t *work;
  // general-path histograms: counts, then the masses as three 11-bit parts
  // (REDs only; part sums stay below 2^32 for rows of up to 2^21 ids), which
  // the planner turns into 64-bit inclusive prefixes stored over the parts
  uint32_t *l1c, *l1p;
  uint64_t *l1m;
  uint32_t *refc, *refp;
  uint64_t *refm;
  SortScratch gsort;
};

__device__ __forceinline__ Layout make_layout(uint8_t *smem, const Plan &pl) {
  Layout L;
  L.data = smem;
  L.work = smem + pl.off_work;
  L.skip = L.work;
  L.seen = pl.seen_map ? reinterpret_cast<uint32_t *>(L.work + pl.map_bytes) : nullptr;
  uint8_t *const maps_end = L.work + pl.map_bytes * (pl.seen_map ? 2 : 1);
  L.ht = reinterpret_cast<int2 *>(maps_end);
  L.queue = reinterpret_cast<int *>(maps_end + pl.ht_cap * 8);
  L.spec = reinterpret_cast<Cand *>(smem + pl.off_spec);
  L.lcand = reinterpret_cast<Cand *>(smem + pl.off_lcand);
  L.bias_id = reinterpret_cast<int32_t *>(smem + pl.off_bias);
  L.bias_val = reinterpret_cast<float *>(smem + pl.off_bias + BIAS_SMEM * 4);
  // general-path area: after the skip bitmap and the seen map (which every
  // scan still reads), over the hash table and the first scan's queue, dead
  // by then
  uint8_t *g = maps_end;
  L.l1c = reinterpret_cast<uint32_t *>(g);
  L.l1p = reinterpret_cast<uint32_t *>(g + NBIN * 4);
  L.l1m = reinterpret_cast<uint64_t *>(g + NBIN * 4);
  uint8_t *gr = g + HIST_BYTES;
  L.refc = reinterpret_cast<uint32_t *>(gr);
  L.refp = reinterpret_cast<uint32_t *>(gr + NBIN * 4);
  L.refm = reinterpret_cast<uint64_t *>(gr + NBIN * 4);
  L.gsort.mid = reinterpret_cast<Cand *>(gr);  // aliases REF
  L.gsort.tmp = reinterpret_cast<uint32_t *>(gr + GCAP * 8);
  L.gsort.S = reinterpret_cast<uint64_t *>(gr + GCAP * 12);
  L.gsort.bcnt = reinterpret_cast<uint32_t *>(gr + GCAP * 20);
  L.gsort.boff = reinterpret_cast<uint32_t *>(gr + GCAP * 20 + GBK * 4);
  L.gsort.in = reinterpret_cast<Cand *>(g + 2 * HIST_BYTES);
  return L;
}

__device__ __forceinline__ uint32_t ht_hash(uint32_t k, int cap) {
  return (k * 2654435761u) & (uint32_t)(cap - 1);
}

// Count word flag: the special position is also disallowed by the mask.
constexpr int HT_MASKED = 1 << 30;

// Insert element position e (row-relative) with count increment c; `slot`
// receives the entry.  Returns 1 if this call created the entry, 0 if it
// existed, -1 if the table is full.
__device__ __forceinline__ int ht_insert(int2 *ht, int cap, int e, int c, int &slot) {
  uint32_t h = ht_hash((uint32_t)e, cap);
  for (int probe = 0; probe < cap; ++probe) {
    // a key never changes once set: seen already, it needs no compare-and-swap
    const int seen = *reinterpret_cast<volatile int *>(&ht[h].x);
    if (seen == e) {
      if (c) atomicAdd(&ht[h].y, c);
      slot = (int)h;
      return 0;
    }
    if (seen != -1) {
      h = (h + 1) & (uint32_t)(cap - 1);
      continue;
    }
    const int prev = atomicCAS(&ht[h].x, -1, e);
    if (prev == -1 || prev == e) {
      if (c) atomicAdd(&ht[h].y, c);
      slot = (int)h;
      return prev == -1 ? 1 : 0;
    }
    h = (h + 1) & (uint32_t)(cap - 1);
  }
  return -1;
}

__device__ __forceinline__ int ht_find(const int2 *ht, int cap, int e) {
  uint32_t h = ht_hash((uint32_t)e, cap);
  for (int probe = 0; probe < cap; ++probe) {
    const int k = ht[h].x;
    if (k == e) return (int)h;
    if (k == -1) return -1;
    h = (h + 1) & (uint32_t)(cap - 1);
  }
  return -1;
}

__device__ __forceinline__ uint32_t allowed32(const uint32_t *aw, int64_t nwords, int64_t g) {
  const int64_t w = g >> 5;
  const int sh = (int)(g & 31);
  const uint32_t lo = w < nwords ? aw[w] : 0u;
  const uint32_t hi = (sh && w + 1 < nwords) ? aw[w + 1] : 0u;
  return sh ? ((lo >> sh) | (hi << (32 - sh))) : lo;
}

// State updates + scalar outputs for one row (called by one thread).
__device__ __forceinline__ void write_row_outputs(const mstar_sampler_params_t &p, int row, int slot, uint32_t token,
                                                  uint32_t status) {
  if (p.stop_ids) {
    const int32_t *st = p.stop_ids + (int64_t)slot * p.NS;
    bool hit = false;
    for (int i = 0; i < p.NS; ++i) hit |= st[i] >= 0 && (uint32_t)st[i] == token;
    if (hit) {
      status |= MSTAR_STATUS_STOP;
      if (p.stop_flags) p.stop_flags[slot] = 1;
    }
  }
  if (p.out_ids) p.out_ids[row] = (int64_t)token;
  if (p.out_ids32) p.out_ids32[row] = (int32_t)token;
  if (p.out_status) p.out_status[row] = (int32_t)status;
  if ((p.flags & MSTAR_FLAG_ADVANCE_OFFSET) && p.offset && !p.uniforms) p.offset[slot] += 1;
  if ((p.flags & MSTAR_FLAG_UPDATE_HISTORY) && p.hist_ids && p.hist_len && p.H > 0) {
    const int32_t len = p.hist_len[slot];
    p.hist_ids[(int64_t)slot * p.H + (len % p.H)] = (int32_t)token;
    p.hist_len[slot] = len + 1;
  }
  if ((p.flags & MSTAR_FLAG_UPDATE_SEEN) && p.seen_bits && (int64_t)(token >> 5) < p.seen_words) {
    atomicOr(&p.seen_bits[(int64_t)slot * p.seen_words + (token >> 5)], 1u << (token & 31));
  }
}

// ------------------------------------------------------------- the tail
//
// The candidate tail runs on all NT threads of one CTA: gather the
// candidates as (order key, weight) pairs, sort them by key, then resolve
// top_k / top_p / the inverse-CDF draw from exact u64 prefix sums of the
// fixed-point weights.  The value-A predicate (positive weight, min_p) is
// monotone in x, so candidates that fail it (weight 0) sort behind every
// candidate that passes: the A set is the first `npass` ranks.

struct TailScr {
  uint64_t *K;   // [TAIL_CAP] order key per candidate (gathered order)
  uint64_t *W;   // [TAIL_CAP] weight per candidate (0 = fails the predicate)
  uint32_t *P;   // [TAIL_CAP] bucket << 16 | position, then rank
  uint64_t *RK;  // [TAIL_CAP] keys: bucket order, then rank order
  uint64_t *RW;  // [TAIL_CAP] weights: bucket order, then rank order
  uint64_t *RS;  // [TAIL_CAP] exclusive weight prefix in rank order
  uint32_t *bc;  // [NBK] bucket counts -> inclusive prefix
  uint64_t *bm;  // [NBK] bucket masses -> inclusive prefix
};

__device__ __forceinline__ TailScr tail_scratch(uint8_t *base) {
  TailScr t;
  t.K = reinterpret_cast<uint64_t *>(base);
  t.W = reinterpret_cast<uint64_t *>(base + TAIL_CAP * 8);
  t.RK = reinterpret_cast<uint64_t *>(base + TAIL_CAP * 16);
  t.RW = reinterpret_cast<uint64_t *>(base + TAIL_CAP * 24);
  t.RS = reinterpret_cast<uint64_t *>(base + TAIL_CAP * 32);
  t.P = reinterpret_cast<uint32_t *>(base + TAIL_CAP * 40);
  t.bc = reinterpret_cast<uint32_t *>(base + TAIL_CAP * 44);
  t.bm = reinterpret_cast<uint64_t *>(base + TAIL_CAP * 44 + NBK * 4);
  return t;
}

__device__ __forceinline__ int tail_log2_buckets(int n) {
  int nbl = 6;
  while (nbl < NBK_LOG2 && (1 << nbl) < 2 * n) ++nbl;
  return nbl;
}

// Called before the barrier that precedes tail_gather.
__device__ __forceinline__ void tail_reset(CtaSh &sh) {
  sh.kmin = ~0ull;
  sh.kmax = 0ull;
  sh.npass = 0u;
  sh.cnt_k = 0u;
}

// Per-thread part of the gather: key and weight of one candidate.
__device__ __forceinline__ void tail_put(const Row &r, float m, uint32_t km, const Cand &cd, int i,
                                         const TailScr &s, uint64_t &kmn, uint64_t &kmx, uint32_t &np) {
  const uint64_t k = ckey(km, cd.x, cd.gid);
  const uint64_t w = weight_A(r, cd.x, m);
  s.K[i] = k;
  s.W[i] = w;
  kmn = u64min(kmn, k);
  kmx = u64max(kmx, k);
  np += w != 0;
}

// Gather epilogue: key range, pass count, cleared buckets.  Block-wide;
// ends with a barrier.
__device__ __forceinline__ void tail_gather_end(uint64_t kmn, uint64_t kmx, uint32_t np, const TailScr &s,
                                                CtaSh &sh) {
  for (int o = 16; o; o >>= 1) {
    kmn = u64min(kmn, (uint64_t)__shfl_xor_sync(~0u, (unsigned long long)kmn, o));
    kmx = u64max(kmx, (uint64_t)__shfl_xor_sync(~0u, (unsigned long long)kmx, o));
  }
  np = __reduce_add_sync(~0u, np);
  if ((threadIdx.x & 31) == 0) {
    if (np) atomicAdd(&sh.npass, np);
    if (kmn <= kmx) {
      atomicMin((unsigned long long *)&sh.kmin, (unsigned long long)kmn);
      atomicMax((unsigned long long *)&sh.kmax, (unsigned long long)kmx);
    }
  }
  for (int b = threadIdx.x; b < NBK; b += NT) {
    s.bc[b] = 0;
    s.bm[b] = 0;
  }
  __syncthreads();
}

// Sort the n gathered candidates (distinct keys) by key ascending: bucket
// counts / masses over the keys' actual range, one scan, scatter, rank inside
// each bucket.  Leaves keys, weights and exclusive weight prefixes in rank
// order in RK / RW / RS.  Block-wide; ends with a barrier.
__device__ void tail_sort(int n, const TailScr &s, CtaSh &sh) {
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int nbl = tail_log2_buckets(n);
  const int NB = 1 << nbl;
  const uint64_t kmin = sh.kmin;
  const uint64_t range = sh.kmax - kmin;
  const int bits = range ? 64 - __clzll((long long)range) : 0;
  const int bsh = bits > nbl ? bits - nbl : 0;
  // bucket masses accumulate as split 32-bit words over the bm array's memory
  uint32_t *mlo = reinterpret_cast<uint32_t *>(s.bm), *mhi = mlo + NBK;
  for (int i = t; i < n; i += NT) {
    const uint32_t b = (uint32_t)((s.K[i] - kmin) >> bsh);
    const uint32_t pos = atomicAdd(&s.bc[b], 1u);
    add_u64_split(&mlo[b], &mhi[b], s.W[i]);
    s.P[i] = (b << 16) | pos;
  }
  __syncthreads();
  {  // inclusive scans of counts and masses; NBK / NT buckets per thread
    constexpr int PER = NBK / NT;
    const int b0 = t * PER;
    uint32_t c = 0, cb[PER];
    uint64_t mm = 0, mb[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      cb[j] = b0 + j < NB ? s.bc[b0 + j] : 0u;
      mb[j] = b0 + j < NB ? get_u64_split(&mlo[b0 + j], &mhi[b0 + j]) : 0ull;
      c += cb[j];
      mm += mb[j];
    }
    uint32_t ic = c;
    uint64_t im = mm;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t uc = __shfl_up_sync(~0u, ic, o);
      const uint64_t um = __shfl_up_sync(~0u, (unsigned long long)im, o);
      if (lane >= o) {
        ic += uc;
        im += um;
      }
    }
    if (lane == 31) {
      sh.red_u32[wid] = ic;
      sh.red_u64[wid] = im;
    }
    __syncthreads();
    uint32_t wc = lane < NWARP ? sh.red_u32[lane] : 0u;
    uint64_t wm = lane < NWARP ? sh.red_u64[lane] : 0ull;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t uc = __shfl_up_sync(~0u, wc, o);
      const uint64_t um = __shfl_up_sync(~0u, (unsigned long long)wm, o);
      if (lane >= o) {
        wc += uc;
        wm += um;
      }
    }
    const uint32_t pc = __shfl_sync(~0u, wc, (wid + 31) & 31);
    const uint64_t pm = __shfl_sync(~0u, (unsigned long long)wm, (wid + 31) & 31);
    uint32_t oc = (wid ? pc : 0u) + ic - c;
    uint64_t om = (wid ? pm : 0ull) + im - mm;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (b0 + j < NB) {  // every thread read its split words before the barrier above
        oc += cb[j];
        om += mb[j];
        s.bc[b0 + j] = oc;
        s.bm[b0 + j] = om;
      }
  }
  __syncthreads();
  for (int i = t; i < n; i += NT) {  // bucket order
    const uint32_t b = s.P[i] >> 16, pos = s.P[i] & 0xFFFFu;
    const uint32_t lo = b ? s.bc[b - 1] : 0u;
    s.RK[lo + pos] = s.K[i];
    s.RW[lo + pos] = s.W[i];
  }
  __syncthreads();
  for (int i = t; i < n; i += NT) {  // rank inside the bucket
    const uint32_t b = s.P[i] >> 16;
    const uint32_t lo = b ? s.bc[b - 1] : 0u, hi = s.bc[b];
    const uint64_t key = s.K[i];
    uint32_t rin = 0;
    uint64_t before = b ? s.bm[b - 1] : 0ull;
    for (uint32_t j = lo; j < hi; ++j) {
      if (s.RK[j] < key) {
        ++rin;
        before += s.RW[j];
      }
    }
    s.P[i] = lo + rin;
    s.RS[lo + rin] = before;
  }
  __syncthreads();
  for (int i = t; i < n; i += NT) {  // keys and weights into rank order
    s.RK[s.P[i]] = s.K[i];
    s.RW[s.P[i]] = s.W[i];
  }
  __syncthreads();
}

// Sort of a small gathered set (n <= 256, distinct keys) by pairwise
// counting: G = NT / slots threads per candidate (8, 4 or 2 for up to 64, 128
// or 256 candidates) each compare it with every
// G-th key (interleaved, conflict-free reads) and sum the counts and the
// weights of the smaller keys, which give its rank and its exclusive weight
// prefix in one pass.  Same outputs as tail_sort (RK / RW / RS in rank
// order).  Block-wide; ends with a barrier.
__device__ void tail_rank_sort(int n, const TailScr &s) {
  const int t = threadIdx.x;
  const int G = n <= 64 ? NT / 64 : n <= 128 ? NT / 128 : NT / 256;
  const int e = t / G, part = t % G;
  const uint64_t key = e < n ? s.K[e] : ~0ull;
  uint32_t c = 0;
  uint64_t before = 0;
#pragma unroll 4
  for (int j = part; j < n; j += G) {  // branch-free: loads of later j overlap
    const bool lt = s.K[j] < key;
    const uint64_t wj = s.W[j];
    c += lt ? 1u : 0u;
    before += lt ? wj : 0ull;
  }
  for (int o = G >> 1; o; o >>= 1) {
    c += __shfl_xor_sync(~0u, c, o);
    before += (uint64_t)__shfl_xor_sync(~0u, (unsigned long long)before, o);
  }
  if (part == 0 && e < n) {
    s.RK[c] = key;
    s.RW[c] = s.W[e];
    s.RS[c] = before;
  }
  __syncthreads();
}

// top_k, top_p and the inverse-CDF draw over the rank-ordered candidates
// (sh.npass of them pass the predicate).  Writes res.token / WK / ckK.
// Block-wide; ends with a barrier.
__device__ void tail_resolve(const Row &r, float u, const TailScr &s, CtaSh &sh) {
  const int t = threadIdx.x;
  const int np = (int)sh.npass;
  const int nA = r.topk ? min(np, r.K) : np;
  if (nA <= 0) {  // no candidate carries weight: the leading one stands
    if (t == 0) {
      sh.res.token = (uint32_t)(s.RK[0] & 0xFFFFFFFFu);
      sh.res.WK = 0;
      sh.res.ckK = s.RK[0];
    }
    __syncthreads();
    return;
  }
  int nK = nA;
  if (r.topp) {  // kept ranks: j == 0 or S_j < P * W_A (a prefix)
    const double thr = __dmul_rn((double)r.P, (double)(s.RS[nA - 1] + s.RW[nA - 1]));
    uint32_t c = 0;
    for (int j = t; j < nA; j += NT) c += (double)s.RS[j] < thr;
    c = __reduce_add_sync(~0u, c);
    if ((t & 31) == 0 && c) atomicAdd(&sh.cnt_k, c);
    __syncthreads();
    nK = max((int)sh.cnt_k, 1);
  }
  const uint64_t WK = s.RS[nK - 1] + s.RW[nK - 1];
  const uint64_t rr = draw_point(u, WK);
  for (int j = t; j < nK; j += NT)
    if (s.RS[j] <= rr && rr < s.RS[j] + s.RW[j]) sh.res.token = (uint32_t)(s.RK[j] & 0xFFFFFFFFu);
  if (t == 0) {
    sh.res.WK = WK;
    sh.res.ckK = s.RK[nK - 1];
  }
  __syncthreads();
}

// tail_resolve for at most NT rank-ordered candidates, by one full
// warp with ballots and reductions (no block barrier).
__device__ void tail_resolve_warp(const Row &r, float u, const TailScr &s, CtaSh &sh) {
  const int lane = threadIdx.x & 31;
  const int np = (int)sh.npass;
  const int nA = r.topk ? min(np, r.K) : np;
  if (nA <= 0) {  // no candidate carries weight: the leading one stands
    if (lane == 0) {
      sh.res.token = (uint32_t)(s.RK[0] & 0xFFFFFFFFu);
      sh.res.WK = 0;
      sh.res.ckK = s.RK[0];
    }
    return;
  }
  int nK = nA;
  if (r.topp) {  // kept ranks: j == 0 or S_j < P * W_A (a prefix)
    const double thr = __dmul_rn((double)r.P, (double)(s.RS[nA - 1] + s.RW[nA - 1]));
    uint32_t c = 0;
    for (int j = lane; j < nA; j += 32) c += (double)s.RS[j] < thr;
    nK = max((int)__reduce_add_sync(~0u, c), 1);
  }
  const uint64_t WK = s.RS[nK - 1] + s.RW[nK - 1];
  const uint64_t rr = draw_point(u, WK);
  for (int j = lane; j < nK; j += 32)
    if (s.RS[j] <= rr && rr < s.RS[j] + s.RW[j]) sh.res.token = (uint32_t)(s.RK[j] & 0xFFFFFFFFu);
  if (lane == 0) {
    sh.res.WK = WK;
    sh.res.ckK = s.RK[nK - 1];
  }
}

// TP shard record: the A set in order (top_k-limited) as (x bits, id)
// pairs.  Block-wide; ends with a barrier.
__device__ void tail_emit(const Row &r, uint32_t km, int tp_cap, uint32_t *rec, const TailScr &s, CtaSh &sh) {
  const int np = (int)sh.npass;
  const int ne = r.topk ? min(np, r.K) : np;
  if (ne <= tp_cap) {
    for (int j = threadIdx.x; j < ne; j += NT) {
      rec[4 + 2 * j] = __float_as_uint(okey_inv(km - (uint32_t)(s.RK[j] >> 32)));
      rec[5 + 2 * j] = (uint32_t)(s.RK[j] & 0xFFFFFFFFu);
    }
  }
  if (threadIdx.x == 0) sh.nemit = ne;
  __syncthreads();
}

// Sort of a larger gathered set (RANK_SMALL < n <= TAIL_CAP) by value
// bucket: 255 buckets uniform in x over the A range below the row max (with
// a margin, so the last bucket holds only values outside A, weight 0, left
// unranked), one counting pass, a warp scan of the counts, a scatter into
// bucket order and a rank inside each bucket; then the exclusive weight
// prefix.  Same outputs as tail_sort (RK / RW / RS in rank order).  Returns
// false, having sorted nothing, when a bucket of A holds more than
// BUCKET_MAX candidates (long runs of exact ties: the caller then sorts by
// order key, whose buckets split ties by id).  A bucket's rank pass costs its
// size per candidate; 256 keeps rows of 1-2 thousand candidates packed into
// a narrow min_p span on this path (a 64 limit sent them to the order-key
// sort: a mixed batch with one such row measured 34.0 -> 26.3 us per step).
// Block-wide; ends with a barrier.
constexpr int RANK_SMALL = 128;
constexpr int RESOLVE_WARP_MAX = 64;  // candidates one warp resolves faster than the whole block
constexpr uint32_t BUCKET_MAX = 256;
__device__ bool tail_bucket_sort(const Row &r, uint32_t km, int n, const TailScr &s, CtaSh &sh) {
  const int t = threadIdx.x, lane = t & 31;
  const float m = okey_inv(km);
  const float span = fmaxf(r.minp ? fminf(23.5f, __fadd_rn(-r.lnMp, 0.25f)) : 23.5f, 1e-3f);
  const float sc = 256.0f / span;
  auto bucket_of = [&](uint64_t key) {  // monotone in the key
    const float x = okey_inv(km - (uint32_t)(key >> 32));
    const float g = __fmul_rn(__fsub_rn(m, x), sc);
    return g >= 255.0f ? 255u : (g > 0.0f ? (uint32_t)g : 0u);
  };
  uint32_t *cnt = s.bc, *start = s.bc + 256;
  uint64_t *BK = s.RS, *BW = s.bm;  // bucket order (RS is written last)
  if (t < 256) cnt[t] = 0u;
  __syncthreads();
  for (int i = t; i < n; i += NT) {
    const uint32_t b = bucket_of(s.K[i]);
    s.P[i] = (b << 16) | atomicAdd(&cnt[b], 1u);
  }
  __syncthreads();
  if (t < 32) {  // exclusive scan of the counts, 8 buckets per lane
    uint32_t c[8], tot = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      c[q] = cnt[lane * 8 + q];
      tot += c[q];
    }
    uint32_t inc = tot;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(~0u, inc, o);
      if (lane >= o) inc += v;
    }
    uint32_t run = inc - tot, big = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      start[lane * 8 + q] = run;
      run += c[q];
      big |= (lane * 8 + q < 255 && c[q] > BUCKET_MAX) ? 1u : 0u;
    }
    big = __reduce_or_sync(~0u, big);
    if (lane == 0) sh.bcast_i = (int)big;
  }
  __syncthreads();
  if (sh.bcast_i) return false;  // uniform
  // with top_k only the first K ranks are read: buckets starting at or past
  // rank K are neither placed nor ranked
  const uint32_t lim = r.topk ? (uint32_t)r.K : 0xFFFFFFFFu;
  for (int i = t; i < n; i += NT) {
    const uint32_t pb = s.P[i];
    if (start[pb >> 16] >= lim) continue;
    const uint32_t dst = start[pb >> 16] + (pb & 0xFFFFu);
    BK[dst] = s.K[i];
    BW[dst] = s.W[i];
  }
  __syncthreads();
  // placed positions: [0, end of the last bucket that starts before lim)
  uint32_t placed = (uint32_t)n;
  if (lim < (uint32_t)n) {
    int lo = 0, hi = 255;  // the last bucket whose start is < lim (starts are non-decreasing)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (start[mid] < lim) lo = mid;
      else hi = mid - 1;
    }
    placed = start[lo] + cnt[lo];
  }
  for (int q = t; q < (int)placed; q += NT) {  // rank inside the bucket
    const uint64_t key = BK[q];
    const uint32_t b = bucket_of(key);
    const uint32_t st = start[b], en = st + cnt[b];
    uint32_t rk = (uint32_t)q - st;  // outside A: any order
    if (b < 255u) {
      rk = 0;
      for (uint32_t j = st; j < en; ++j) rk += BK[j] < key ? 1u : 0u;
    }
    s.RK[st + rk] = key;
    s.RW[st + rk] = BW[q];
  }
  __syncthreads();
  {  // exclusive prefix of the weights in rank order, a segment per thread
    const int seg = (n + NT - 1) / NT;
    const int a0 = min(n, t * seg), a1 = min(n, a0 + seg);
    uint64_t loc = 0;
    for (int j = a0; j < a1; ++j) loc += s.RW[j];
    uint64_t tot;
    uint64_t run = block_exscan_u64(loc, tot, sh);
    for (int j = a0; j < a1; ++j) {
      s.RS[j] = run;
      run += s.RW[j];
    }
  }
  __syncthreads();
  return true;
}

// Sort the n gathered candidates (tail_put, every thread's kmn / kmx / np)
// into RK / RW / RS rank order; sh.npass counts those passing the value-A
// predicate.  Block-wide; ends with a barrier.
__device__ void tail_sort_gathered(const Row &r, uint32_t km, int n, uint64_t kmn, uint64_t kmx, uint32_t np,
                                   const TailScr &ts, CtaSh &sh) {
  np = __reduce_add_sync(~0u, np);
  if ((threadIdx.x & 31) == 0 && np) atomicAdd(&sh.npass, np);
  __syncthreads();  // keys, weights and the pass count complete
  bool sorted = true;
  if (n <= RANK_SMALL) tail_rank_sort(n, ts);
  else sorted = tail_bucket_sort(r, km, n, ts, sh);
  if (!sorted) {  // long runs of ties: buckets of the order key (the pass count is in already)
    tail_gather_end(kmn, kmx, 0u, ts, sh);
    tail_sort(n, ts, sh);
  }
}

// Sort the n gathered candidates and resolve them (MODE 0: res.token / WK /
// ckK) or emit the shard record (MODE 1).  Block-wide; a small set is
// resolved by warp 0 alone, so callers read sh.res after a barrier.
template <int MODE>
__device__ void tail_finish(const Row &r, float u, uint32_t km, int n, uint64_t kmn, uint64_t kmx, uint32_t np,
                            int tp_cap, uint32_t *rec, const TailScr &ts, CtaSh &sh) {
  tail_sort_gathered(r, km, n, kmn, kmx, np, ts, sh);
  if (MODE == 0) {
    if (n <= RESOLVE_WARP_MAX) {  // a few ranks: one warp, no block barrier
      if (threadIdx.x < 32) tail_resolve_warp(r, u, ts, sh);
    } else {
      tail_resolve(r, u, ts, sh);
    }
  } else {
    tail_emit(r, km, tp_cap, rec, ts, sh);
  }
}


// Clears the per-bucket counts and masses tail_finish1 accumulates into;
// called by the leader's threads t0, t0 + stride, ... before a barrier that
// precedes tail_finish1.
__device__ __forceinline__ void tail_clear1(const TailScr &s, int t0, int stride) {
  uint32_t *w = s.bc;  // counts [256]
  for (int i = t0; i < 256; i += stride) w[i] = 0u;
  uint32_t *mw = reinterpret_cast<uint32_t *>(s.bm);  // mass words: lo [256], hi [256]
  for (int i = t0; i < 512; i += stride) mw[i] = 0u;
}

// tail_finish for RANK_SMALL < n <= NT candidates, candidate i held by
// thread i (key, weight; valid = i < n), sorted by value bucket with fewer
// block-wide steps than tail_bucket_sort: each candidate's bucket count and
// weight go into per-bucket counts and masses in one atomic pass (counters
// cleared by tail_clear1 beforehand), one warp scan gives every bucket's
// first rank and exclusive mass, a scatter into bucket order, and a rank
// inside the bucket that also sums the weights of the bucket's smaller keys,
// so each candidate's exclusive weight prefix is its bucket's exclusive
// mass plus that sum: no block-wide prefix scan.  Same outputs and buckets
// as tail_bucket_sort; runs of ties (a bucket of A with more than
// BUCKET_MAX candidates) fall back to the order-key sort.  Block-wide.
template <int MODE>
__device__ void tail_finish1(const Row &r, float u, uint32_t km, int n, bool valid, uint64_t key, uint64_t w,
                             uint64_t kmn, uint64_t kmx, int tp_cap, uint32_t *rec, const TailScr &s, CtaSh &sh) {
  const int t = threadIdx.x, lane = t & 31;
  const float m = okey_inv(km);
  const float span = fmaxf(r.minp ? fminf(23.5f, __fadd_rn(-r.lnMp, 0.25f)) : 23.5f, 1e-3f);
  const float sc = 256.0f / span;
  uint32_t *cnt = s.bc, *start = s.bc + 256;
  uint32_t *mlo = reinterpret_cast<uint32_t *>(s.bm), *mhi = mlo + 256;
  uint64_t *mst = s.bm + 256;       // exclusive bucket masses
  uint64_t *BK = s.K, *BW = s.W;    // bucket order (each key and weight is in its thread's registers)
  uint32_t b = 255u, pos = 0u;
  if (valid) {
    const float x = okey_inv(km - (uint32_t)(key >> 32));
    const float g = __fmul_rn(__fsub_rn(m, x), sc);
    b = g >= 255.0f ? 255u : (g > 0.0f ? (uint32_t)g : 0u);
    pos = atomicAdd(&cnt[b], 1u);
    if (w) add_u64_split(&mlo[b], &mhi[b], w);
  }
  const uint32_t np = __reduce_add_sync(~0u, (valid && w != 0) ? 1u : 0u);
  if (lane == 0 && np) atomicAdd(&sh.npass, np);
  __syncthreads();  // counts, masses and the pass count complete
  if (t < 32) {  // exclusive scans of the counts and masses, 8 buckets per lane
    uint32_t c[8], tot = 0;
    uint64_t ms[8], mt = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int bq = lane * 8 + q;
      c[q] = cnt[bq];
      ms[q] = get_u64_split(&mlo[bq], &mhi[bq]);
      tot += c[q];
      mt += ms[q];
    }
    uint32_t inc = tot;
    uint64_t minc = mt;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(~0u, inc, o);
      const uint64_t mv = __shfl_up_sync(~0u, (unsigned long long)minc, o);
      if (lane >= o) {
        inc += v;
        minc += mv;
      }
    }
    uint32_t run = inc - tot, big = 0;
    uint64_t mrun = minc - mt;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      start[lane * 8 + q] = run;
      mst[lane * 8 + q] = mrun;
      run += c[q];
      mrun += ms[q];
      big |= (lane * 8 + q < 255 && c[q] > BUCKET_MAX) ? 1u : 0u;
    }
    big = __reduce_or_sync(~0u, big);
    if (lane == 0) sh.bcast_i = (int)big;
  }
  __syncthreads();  // bucket starts and masses
  if (sh.bcast_i) {  // uniform: long runs of ties, the order-key sort (keys and weights gathered by the caller)
    tail_gather_end(kmn, kmx, 0u, s, sh);
    tail_sort(n, s, sh);
  } else {
    // with top_k only the first K ranks are read: buckets starting at or
    // past rank K are neither placed nor ranked
    const uint32_t lim = r.topk ? (uint32_t)r.K : 0xFFFFFFFFu;
    const uint32_t st = start[b];
    const bool placed = valid && st < lim;
    if (placed) {
      BK[st + pos] = key;
      BW[st + pos] = w;
    }
    __syncthreads();  // bucket order
    if (placed) {
      uint32_t rk = pos;  // outside A: any order
      uint64_t before = 0;
      if (b < 255u) {
        rk = 0;
        const uint32_t en = st + cnt[b];
        for (uint32_t j = st; j < en; ++j) {
          const bool lt = BK[j] < key;
          rk += lt ? 1u : 0u;
          before += lt ? BW[j] : 0ull;
        }
      }
      s.RK[st + rk] = key;
      s.RW[st + rk] = w;
      s.RS[st + rk] = mst[b] + before;
    }
    __syncthreads();  // rank order
  }
  if (MODE == 0) {
    tail_resolve(r, u, s, sh);  // (more than RANK_SMALL candidates: one rank per thread)
  } else {
    tail_emit(r, km, tp_cap, rec, s, sh);
  }
}

// ------------------------------------------------------------ the kernel

// What the out-of-line paths (general rounds, dense debug outputs) share
// with the kernel body.
struct RowCtx {
  const mstar_sampler_params_t *p;
  const Plan *pl;
  Layout L;
  Slice sl;
  Row r;
  const uint8_t *rowp;
  float m, theta, u;
  uint32_t km;
  int nspec, rank, S, row, slot;
  int64_t c0, c1, gbase;
  uint32_t *rec;  // TP shard record (MODE 1)
  bool empty;
};

__device__ __forceinline__ float xform(const Row &r, float v) { return r.greedy ? v : __fmul_rn(v, r.invT); }

// Value bins of the general path's first histogram: bin b holds the values x
// with E(b+1) < x <= E(b), E(b) = m - b * w (binary32 operations, so every CTA
// and the planner agree on every bin), w = (m - theta) / NBIN.  Bins uniform
// in value keep the bins near the row max (where the mass is) narrow; bins
// of the order key itself would give almost all of them to values near zero.
// The bins are monotone in the order key, so each is a key range.
struct VBins {
  float m, w, iw;  // row max, bin width, an approximate 1 / w (first guess only)
};
__device__ __forceinline__ float vb_edge(const VBins &v, int b) { return __fsub_rn(v.m, __fmul_rn((float)b, v.w)); }
__device__ __forceinline__ int vb_bin(const VBins &v, float x) {
  const float g = __fmul_rn(__fsub_rn(v.m, x), v.iw);
  int b = g >= (float)(NBIN - 1) ? NBIN - 1 : (g > 0.0f ? (int)g : 0);
  while (b > 0 && x > vb_edge(v, b)) --b;
  while (b < NBIN - 1 && !(x > vb_edge(v, b + 1))) ++b;
  return b;
}
// The first of NBIN bins (counts in hist, from the top) at which the count
// from the top reaches K, or NBIN - 1 if none does.  One full warp; every
// lane returns the same bin.
__device__ __forceinline__ int vb_kbin(const uint32_t *hist, uint32_t K) {
  static_assert(NBIN == 32 * 32, "32 chunks of 32 bins");
  const int lane = threadIdx.x & 31;
  // lane l sums chunk l (bins 32 l .. 32 l + 31), reading them in a rotated
  // order so that the 32 lanes hit 32 different banks at every step
  uint32_t s = 0;
#pragma unroll 8
  for (int i = 0; i < 32; ++i) s += hist[lane * 32 + ((i + lane) & 31)];
  uint32_t inc = s;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(~0u, inc, o);
    if (lane >= o) inc += t;
  }
  const unsigned reach = __ballot_sync(~0u, inc >= K);
  if (!reach) return NBIN - 1;
  const int ch = __ffs(reach) - 1;  // the chunk where the count reaches K
  const uint32_t before = __shfl_sync(~0u, inc - s, ch);
  uint32_t ci = hist[ch * 32 + lane];  // then its bins, one per lane
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(~0u, ci, o);
    if (lane >= o) ci += t;
  }
  const unsigned rb = __ballot_sync(~0u, before + ci >= K);
  return ch * 32 + (__ffs(rb) - 1);
}

// Order-key range [lo, hi] of value bin b (clipped to the A range's keys <= kmax).
__device__ __forceinline__ void vb_range(const VBins &v, uint32_t km, int b, uint64_t kmax, uint64_t &lo,
                                         uint64_t &hi) {
  lo = b == 0 ? 0ull : (uint64_t)(km - okey(vb_edge(v, b))) << 32;
  hi = b == NBIN - 1 ? kmax : ((uint64_t)(km - okey(vb_edge(v, b + 1))) << 32) - 1ull;
  hi = u64min(hi, kmax);
  lo = u64min(lo, kmax + 1);
}

// General path: leader-driven rounds of histogram (count + mass) and
// compaction over the still-resident slices until every boundary (top_k,
// top_p, the draw) is pinned to a bin small enough to sort.  Executed by
// every CTA of the cluster.
template <typename T, int MODE>
__device__ __forceinline__ void general_path(const RowCtx &c, CtaSh &sh) {
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, lane = tid & 31;
  const int rank = c.rank, S = c.S;
  const Layout &L = c.L;
  const Slice &sl = c.sl;
  const Row &r = c.r;
  const Plan &pl = *c.pl;
  const float m = c.m, theta = c.theta, u = c.u;
  const uint32_t km = c.km;
  const int nspec = c.nspec;
  uint32_t *rec = c.rec;
  Planner &P = sh.pl;
  // this CTA's values above its own threshold (counted by the first pass)
  const uint32_t seen = sh.scanned ? sh.scanned * (uint32_t)Elem<T>::VEC : (uint32_t)sl.nvec * Elem<T>::VEC;
  const bool dense_l1 = sh.nloc * 4u > seen;
  VBins vb;
  vb.m = m;
  vb.w = __fmul_rn(__fsub_rn(m, theta), 1.0f / NBIN);
  vb.iw = 1.0f / vb.w;
  // value bins unless the width is not a positive finite number
  const bool vbins = vb.w > 0.0f && vb.w < INFINITY && vb.iw < INFINITY;
  if (rank == 0 && tid == 0) {
    memset(&P, 0, sizeof(P));
    P.state = ST_START;
    sh.res.status |= MSTAR_STATUS_GENERAL;
    tail_reset(sh);
  }
  for (int round = 0; round < MAX_ROUNDS; ++round) {
    if (rank == 0) {
      // ================= leader planning (block-wide) =================
      for (int guard = 0; guard < 16; ++guard) {
        __syncthreads();
        const int state = P.state;
        __syncthreads();
        if (state == ST_START) {
          if (tid == 0) {
            const uint32_t DA = km - okey(theta);
            P.l1lo = 0;
            P.l1hi = ((uint64_t)DA << 32) | 0xFFFFFFFFull;
            if (vbins) {  // value bins (shift -1 marks them)
              P.l1shift = -1;
              P.l1nbins = NBIN;
            } else {
              const int bits = 64 - __clzll((long long)(P.l1hi - P.l1lo));
              P.l1shift = bits > NBIN_LOG2 ? bits - NBIN_LOG2 : 0;
              P.l1nbins = (int)((P.l1hi - P.l1lo) >> P.l1shift) + 1;
            }
            sh.cmd = Cmd{OP_HIST, TGT_L1, P.l1lo, P.l1hi, P.l1shift, P.l1nbins};
            P.state = ST_AFTER_L1;
          }
          for (int b = tid; b < NBIN * 4; b += NT) L.l1c[b] = 0;  // counts and parts
          break;
        }
        if (state == ST_AFTER_L1 || state == ST_LOC_AFTER_REF) {
          uint32_t *C = state == ST_AFTER_L1 ? L.l1c : L.refc;
          uint64_t *M = state == ST_AFTER_L1 ? L.l1m : L.refm;
          const uint32_t *Mp = state == ST_AFTER_L1 ? L.l1p : L.refp;
          constexpr int PER = NBIN / NT;
          uint64_t lc[PER], lm[PER], sc = 0, sm = 0;
#pragma unroll
          for (int q = 0; q < PER; ++q) {  // read before the scan's barriers; M is written over the parts
            const int b = tid * PER + q;
            lc[q] = C[b];
            lm[q] = (uint64_t)Mp[b] + ((uint64_t)Mp[NBIN + b] << 11) + ((uint64_t)Mp[2 * NBIN + b] << 22);
            sc += lc[q];
            sm += lm[q];
          }
          uint64_t oc, om, tc, tm;
          block_exscan2_u64(sc, sm, oc, om, tc, tm, sh);
#pragma unroll
          for (int q = 0; q < PER; ++q) {
            oc += lc[q];
            om += lm[q];
            C[tid * PER + q] = (uint32_t)oc;
            M[tid * PER + q] = om;
          }
          if (tid == 0) sh.bcast_i = -1;
          __syncthreads();
          if (state == ST_AFTER_L1) {
            if (r.topk && tc > (uint64_t)r.K) {  // the L1 bin holding the K-th key (prefixes are monotone)
              const uint32_t km1 = (uint32_t)(r.K - 1);
              for (int b = tid; b < P.l1nbins; b += NT)
                if (C[b] > km1 && (b == 0 || C[b - 1] <= km1)) sh.bcast_i = b;
              __syncthreads();
            }
            if (tid == 0) {
              P.N = tc;
              P.Wv = tm;
              P.level = 0;
              P.lo = P.l1lo;
              P.hi = P.l1hi;
              P.shift = P.l1shift;
              P.nbins = P.l1nbins;
              P.base_c = 0;
              P.base_m = 0;
              const bool needA = r.topk && P.N > (uint64_t)r.K;
              const int b_end = needA && sh.bcast_i >= 0 ? sh.bcast_i : P.nbins - 1;
              const uint64_t pre = L.l1c[b_end];
              if (pre <= (uint64_t)TAIL_CAP) {
                uint64_t blo, bhi;
                if (P.l1shift < 0) vb_range(vb, km, b_end, P.l1hi, blo, bhi);
                else bhi = u64min(P.l1hi, P.l1lo + (((uint64_t)b_end + 1) << P.l1shift) - 1);
                sh.cmd = Cmd{OP_COMPACT, 0, P.l1lo, bhi, 0, 0};
                P.state = ST_AFTER_PREFIX;
              } else if (needA) {
                P.stage = 0;
                P.qkind = Q_COUNT;
                P.tcount = (uint64_t)(r.K - 1);
                P.state = ST_LOC_BIN;
              } else if (MODE == 1) {
                P.state = ST_FINISH;
                sh.tp_ovf = 1;
              } else {
                P.WA = P.Wv;
                P.ckA = P.l1hi;
                P.stage = 1;
                if (r.topp) {
                  P.thr = __dmul_rn((double)r.P, (double)P.WA);
                  if (!(0.0 < P.thr)) {
                    P.qkind = Q_COUNT;
                    P.tcount = 0;
                  } else {
                    P.qkind = Q_LASTLT;
                  }
                } else {
                  P.WK = P.WA;
                  P.ckK = P.ckA;
                  P.stage = 2;
                  P.qkind = Q_POINT;
                  P.tpoint = draw_point(u, P.WK);
                }
                P.state = ST_LOC_BIN;
              }
            }
            __syncthreads();
            if (P.state == ST_AFTER_PREFIX) break;
            continue;
          }
          if (tid == 0) {
            P.level = 1;
            P.state = ST_LOC_BIN;
          }
          continue;
        }
        if (state == ST_LOC_BIN) {
          const uint32_t *C = P.level == 0 ? L.l1c : L.refc;
          const uint64_t *M = P.level == 0 ? L.l1m : L.refm;
          if (tid == 0) sh.bcast_i = -1;
          __syncthreads();
          for (int b = tid; b < P.nbins; b += NT) {
            const uint64_t pc0 = P.base_c + (b ? C[b - 1] : 0), pc1 = P.base_c + C[b];
            const uint64_t pm0 = P.base_m + (b ? M[b - 1] : 0), pm1 = P.base_m + M[b];
            bool hit = false;
            if (P.qkind == Q_COUNT) hit = pc0 <= P.tcount && P.tcount < pc1;
            else if (P.qkind == Q_POINT) hit = pm0 <= P.tpoint && P.tpoint < pm1;
            if (hit) sh.bcast_i = b;
            if (P.qkind == Q_LASTLT && pc1 > pc0 && (double)pm0 < P.thr) atomicMax(&sh.bcast_i, b);
          }
          __syncthreads();
          if (tid == 0) {
            const int b = sh.bcast_i;
            if (b < 0) {  // cannot happen for consistent inputs; finish defensively
              P.state = ST_FINISH;
              sh.res.status |= MSTAR_STATUS_EMPTY;
            } else {
              uint64_t blo, bhi;
              if (P.shift < 0) {
                vb_range(vb, km, b, P.hi, blo, bhi);
              } else {
                blo = P.lo + ((uint64_t)b << P.shift);
                bhi = u64min(P.hi, blo + (1ull << P.shift) - 1);
              }
              const uint64_t cnt = (uint64_t)C[b] - (b ? C[b - 1] : 0);
              P.cbase_c = P.base_c + (b ? C[b - 1] : 0);
              P.cbase_m = P.base_m + (b ? M[b - 1] : 0);
              if (cnt <= (uint64_t)GCAP || P.shift == 0 || blo >= bhi) {
                sh.cmd = Cmd{OP_COMPACT, 0, blo, bhi, 0, 0};
                P.state = ST_LOC_AFTER_COMPACT;
              } else {
                P.base_c = P.cbase_c;
                P.base_m = P.cbase_m;
                P.lo = blo;
                P.hi = bhi;
                const int bits = 64 - __clzll((long long)(bhi - blo));
                P.shift = bits > NBIN_LOG2 ? bits - NBIN_LOG2 : 0;
                P.nbins = (int)((bhi - blo) >> P.shift) + 1;
                sh.cmd = Cmd{OP_HIST, TGT_REF, blo, bhi, P.shift, P.nbins};
                P.state = ST_LOC_AFTER_REF;
              }
            }
          }
          __syncthreads();
          if (P.state == ST_LOC_AFTER_REF) {
            for (int b = tid; b < NBIN * 4; b += NT) L.refc[b] = 0;  // counts and parts
          }
          if (P.state == ST_FINISH) continue;
          break;
        }
        if (state == ST_AFTER_PREFIX) {
          if (tid < 32) {  // per-CTA counts of the compacted range
            const uint32_t c = lane < S ? min(cluster.map_shared_rank(&sh, lane)->nloc, (uint32_t)LCAP) : 0u;
            uint32_t inc = c;
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t v = __shfl_up_sync(~0u, inc, o);
              if (lane >= o) inc += v;
            }
            if (lane < 16) {
              sh.goff[lane] = inc - c;
              sh.gcnt[lane] = c;
            }
            const uint32_t tot = __shfl_sync(~0u, inc, 31);
            if (lane == 0) sh.ncand = min(tot, (uint32_t)TAIL_CAP);
          }
          __syncthreads();
          {  // every CTA's compacted list, over DSMEM, into the tail
            const int n = (int)sh.ncand;
            const TailScr ts = tail_scratch(L.data);  // the leader's slice data is dead by now
            uint64_t kmn = ~0ull, kmx = 0ull;
            uint32_t np = 0;
            if (P.l1shift < 0 && n > 64) {
              // Placed by value bin: the first histogram's prefix counts give
              // every bin's slot range in rank order (the compacted prefix is
              // exactly bins 0..b_end), so one pass places each candidate in
              // its bin and a pass over each (narrow) bin ranks it there.
              uint32_t *fill = L.refc;  // per-bin fill counters (the REF histogram is idle here)
              const uint32_t *C = L.l1c;
              for (int b = tid; b < NBIN; b += NT) fill[b] = 0;
              __syncthreads();
              for (int i = tid; i < n; i += NT) {
                int q = 0;
                while (q + 1 < S && i >= (int)sh.goff[q + 1]) ++q;
                const Cand cd = cluster.map_shared_rank(L.lcand, q)[i - (int)sh.goff[q]];
                const int b = vb_bin(vb, cd.x);
                const uint32_t pos = (b ? C[b - 1] : 0u) + atomicAdd(&fill[b], 1u);
                if (pos < (uint32_t)n) {
                  const uint64_t w = weight_A(r, cd.x, m);
                  ts.K[pos] = ckey(km, cd.x, cd.gid);
                  ts.W[pos] = w;
                  ts.P[pos] = (uint32_t)b;
                  np += w != 0;
                }
              }
              np = __reduce_add_sync(~0u, np);
              if (lane == 0 && np) atomicAdd(&sh.npass, np);
              __syncthreads();
              for (int pos = tid; pos < n; pos += NT) {  // rank inside the bin
                const int b = (int)ts.P[pos];
                const uint32_t st = b ? C[b - 1] : 0u, en = min(C[b], (uint32_t)n);
                const uint64_t key = ts.K[pos];
                uint32_t rk = 0;
                for (uint32_t j = st; j < en; ++j) rk += ts.K[j] < key;
                ts.RK[st + rk] = key;
                ts.RW[st + rk] = ts.W[pos];
              }
              __syncthreads();
              {  // exclusive prefix of the weights in rank order
                const int seg = (n + NT - 1) / NT;
                const int a0 = min(n, tid * seg), a1 = min(n, a0 + seg);
                uint64_t loc = 0;
                for (int j = a0; j < a1; ++j) loc += ts.RW[j];
                uint64_t tot;
                uint64_t run = block_exscan_u64(loc, tot, sh);
                for (int j = a0; j < a1; ++j) {
                  ts.RS[j] = run;
                  run += ts.RW[j];
                }
              }
              __syncthreads();
              if (MODE == 0) tail_resolve(r, u, ts, sh);
              else tail_emit(r, km, pl.tp_cap, rec, ts, sh);
            } else {
              for (int i = tid; i < n; i += NT) {  // one candidate per thread; the lists lie gap-free at goff
                int q = 0;
                while (q + 1 < S && i >= (int)sh.goff[q + 1]) ++q;
                const Cand *list = cluster.map_shared_rank(L.lcand, q);
                tail_put(r, m, km, list[i - (int)sh.goff[q]], i, ts, kmn, kmx, np);
              }
              tail_finish<MODE>(r, u, km, n, kmn, kmx, np, pl.tp_cap, rec, ts, sh);
            }
          }
          if (tid == 0) P.state = ST_FINISH;
          __syncthreads();
          continue;
        }
        if (state == ST_LOC_AFTER_COMPACT) {
          if (tid < 32) {  // per-CTA counts of the compacted bin
            const uint32_t c = lane < S ? min(cluster.map_shared_rank(&sh, lane)->nloc, (uint32_t)LCAP) : 0u;
            uint32_t inc = c;
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t v = __shfl_up_sync(~0u, inc, o);
              if (lane >= o) inc += v;
            }
            if (lane < 16) sh.goff[lane] = inc - c;
            if (lane == 31) sh.ncand = min(inc, (uint32_t)GCAP);
          }
          __syncthreads();
          const int n = (int)sh.ncand;
          for (int i = tid; i < n; i += NT) {  // every CTA's list (DSMEM), one element per thread
            int q = 0;
            while (q + 1 < S && i >= (int)sh.goff[q + 1]) ++q;
            L.gsort.in[i] = cluster.map_shared_rank(L.lcand, q)[i - (int)sh.goff[q]];
          }
          __syncthreads();
          if (n <= 128) tail_sort_scan_small(L.gsort.in, n, m, L.gsort);
          else tail_sort_scan(L.gsort.in, n, m, L.gsort, sh);
          const uint64_t *Sx = L.gsort.S;
          const Cand *sorted = L.gsort.in;
          if (tid == 0) sh.bcast_i = -1;
          __syncthreads();
          for (int j = tid; j < n; j += NT) {
            const uint64_t se = P.cbase_m + S_excl(Sx, j), si = P.cbase_m + Sx[j];
            bool hit = false;
            if (P.qkind == Q_COUNT) hit = (P.cbase_c + j) == P.tcount;
            else if (P.qkind == Q_POINT) hit = se <= P.tpoint && P.tpoint < si;
            if (hit) sh.bcast_i = j;
            if (P.qkind == Q_LASTLT && (double)se < P.thr) atomicMax(&sh.bcast_i, j);
          }
          __syncthreads();
          if (tid == 0) {
            const int j = sh.bcast_i;
            if (j < 0) {
              P.state = ST_FINISH;
              sh.res.status |= MSTAR_STATUS_EMPTY;
            } else {
              const uint64_t ck = ckey(km, sorted[j].x, sorted[j].gid);
              const uint64_t si = P.cbase_m + Sx[j];
              P.level = 0;
              P.lo = P.l1lo;
              P.hi = P.l1hi;
              P.shift = P.l1shift;
              P.nbins = P.l1nbins;
              P.base_c = 0;
              P.base_m = 0;
              if (P.stage == 0) {  // A boundary (top_k)
                P.WA = si;
                P.ckA = ck;
                if (MODE == 1 || r.K <= TAIL_CAP) {
                  sh.cmd = Cmd{OP_COMPACT, 0, P.l1lo, ck, 0, 0};
                  P.state = ST_AFTER_PREFIX;
                } else {
                  P.stage = 1;
                  if (r.topp) {
                    P.thr = __dmul_rn((double)r.P, (double)P.WA);
                    if (!(0.0 < P.thr)) {
                      P.qkind = Q_COUNT;
                      P.tcount = 0;
                    } else {
                      P.qkind = Q_LASTLT;
                    }
                  } else {
                    P.WK = P.WA;
                    P.ckK = P.ckA;
                    P.stage = 2;
                    P.qkind = Q_POINT;
                    P.tpoint = draw_point(u, P.WK);
                  }
                  P.state = ST_LOC_BIN;
                }
              } else if (P.stage == 1) {  // top-p boundary: last kept element
                P.WK = si;
                P.ckK = ck;
                P.stage = 2;
                P.qkind = Q_POINT;
                P.tpoint = draw_point(u, P.WK);
                P.state = ST_LOC_BIN;
              } else {  // draw
                sh.res.token = sorted[j].gid;
                sh.res.WK = P.WK;
                sh.res.ckK = P.ckK;
                P.state = ST_FINISH;
              }
            }
          }
          __syncthreads();
          if (P.state == ST_AFTER_PREFIX) break;
          continue;
        }
        if (state == ST_FINISH) {
          if (tid == 0) sh.cmd = Cmd{OP_DONE, 0, 0, 0, 0, 0};
          break;
        }
      }
      __syncthreads();
    }
    cluster.sync();  // command published
    const Cmd cmd = cluster.map_shared_rank(&sh, 0)->cmd;
    if (cmd.op == OP_DONE) break;
    if (cmd.op == OP_HIST) {
      uint32_t *hc = rank == 0 ? (cmd.target == TGT_L1 ? L.l1c : L.refc) : L.l1c;
      uint32_t *hp = hc + NBIN;  // the three mass parts follow the counts
      if (rank != 0) {
        for (int b = tid; b < NBIN * 4; b += NT) hc[b] = 0;
        __syncthreads();
      }
      auto add = [&](float x, uint32_t gid, uint64_t w, bool valid) {
        if (!valid) return;
        const int b = cmd.shift < 0 ? vb_bin(vb, x) : (int)((ckey(km, x, gid) - cmd.lo) >> cmd.shift);
        atomicAdd(&hc[b], 1u);
        const uint32_t p0 = (uint32_t)w & 0x7FFu, p1 = (uint32_t)(w >> 11) & 0x7FFu, p2 = (uint32_t)(w >> 22);
        if (p0) atomicAdd(&hp[b], p0);
        if (p1) atomicAdd(&hp[NBIN + b], p1);
        if (p2) atomicAdd(&hp[2 * NBIN + b], p2);
      };
      // the first histogram spans the whole A range: dense when the first
      // pass found most of this CTA's values above its threshold; the warp
      // lists sit in the CTA-local candidate list, unused by histogram rounds
      int *wq = reinterpret_cast<int *>(L.lcand) + (tid >> 5) * QW;
      if (cmd.target == TGT_L1 && dense_l1)
        for_each_value<T, true>(sl, L.spec, nspec, r, m, theta, cmd.lo, cmd.hi, wq, add);
      else
        for_each_value<T, false>(sl, L.spec, nspec, r, m, theta, cmd.lo, cmd.hi, wq, add);
      if (rank != 0) {
        __syncthreads();
        uint32_t *rc = cluster.map_shared_rank(cmd.target == TGT_L1 ? L.l1c : L.refc, 0);
        for (int b = tid; b < cmd.nbins; b += NT) {
          if (hc[b]) {
            atomicAdd(&rc[b], hc[b]);
#pragma unroll
            for (int q = 1; q <= 3; ++q)
              if (hc[q * NBIN + b]) atomicAdd(&rc[q * NBIN + b], hc[q * NBIN + b]);
          }
        }
      }
    } else {  // OP_COMPACT into the CTA-local list
      if (tid == 0) sh.nloc = 0;
      __syncthreads();
      // the warp lists sit in the REF histogram's area, dead once a bin is being compacted
      for_each_value<T, false>(sl, L.spec, nspec, r, m, theta, cmd.lo, cmd.hi,
                               reinterpret_cast<int *>(L.refc) + (tid >> 5) * QW,
                        [&](float x, uint32_t gid, uint64_t, bool valid) {
                          const uint32_t idx = warp_reserve(&sh.nloc, valid ? 1u : 0u);
                          if (valid && idx < (uint32_t)LCAP) L.lcand[idx] = Cand{x, gid};
                        });
    }
    cluster.sync();  // round results complete
  }
}

// Every position of the slice once through emit(e, x): the final value of
// each id (the resident logits transformed, then the specials' and seen ids'
// final values over them).  Block-wide (one barrier between the two).
template <typename T, typename Emit>
__device__ __forceinline__ void dense_values(const RowCtx &c, Emit &&emit) {
  const mstar_sampler_params_t &p = *c.p;
  const Row &r = c.r;
  const uint32_t *aw = p.allowed_bits ? p.allowed_bits + (int64_t)c.slot * p.allowed_words : nullptr;
  for (int64_t e = c.c0 + threadIdx.x; e < c.c1; e += NT) {
    const float v = Elem<T>::load(c.rowp, e);
    const int64_t g = e + c.gbase;
    const bool allowed = !aw || ((aw[g >> 5] >> (g & 31)) & 1u);
    float x;
    if (v != v) x = v;
    else if (!allowed) x = -INFINITY;
    else x = xform(r, v);
    emit(e, x);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < c.nspec; i += NT) emit((int64_t)c.L.spec[i].gid - c.gbase, c.L.spec[i].x);
  // seen-mask ids from global memory (the leader's resident slice may hold
  // the tail's scratch by now)
  for_each_seen<T>(c.sl, r, true, threadIdx.x, NT, [&](const Cand &cd, bool valid) {
    if (valid) emit((int64_t)cd.gid - c.gbase, cd.x);
  });
}

// Dense debug outputs (x, kept, probs) of this CTA's slice, after the
// barrier that published the leader's result.
template <typename T>
__device__ __forceinline__ void debug_dense(const RowCtx &c, CtaSh &sh) {
  cg::cluster_group cluster = cg::this_cluster();
  const mstar_sampler_params_t &p = *c.p;
  const Row &r = c.r;
  const Result res = cluster.map_shared_rank(&sh, 0)->res;
  const uint32_t kmm = okey(res.m);
  dense_values<T>(c, [&](int64_t e, float x) {
    const int64_t o = (int64_t)c.row * p.V + e;
    const uint32_t gid = (uint32_t)(e + c.gbase);
    bool kept = false;
    float prob = 0.0f;
    if (!res.empty && x == x) {
      if (res.greedy) {
        kept = gid == res.token;
        prob = kept ? 1.0f : 0.0f;
      } else if (x > -INFINITY && x <= res.m && ckey(kmm, x, gid) <= res.ckK && weight_A(r, x, res.m) != 0) {
        // (kept members are members of A: positive weight, past min_p; the
        // last kept key alone does not say that for keys between theta and
        // the A boundary)
        kept = true;
        prob = (float)__ddiv_rn((double)spec_w_from_e(spec_e(x, res.m)), (double)res.WK);
      }
    }
    if (p.out_x) p.out_x[o] = x;
    if (p.out_kept) p.out_kept[o] = kept ? 1 : 0;
    if (p.out_probs) p.out_probs[o] = prob;
  });
}

template <typename T, int MODE>
__global__ void __launch_bounds__(NT, 1)
    sampler_kernel(const mstar_sampler_params_t p, const Plan pl, uint32_t *tp_send) {
  using Acc = typename Elem<T>::Acc;
  constexpr int VEC = Elem<T>::VEC;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int S = pl.S;
  const int row = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ CtaSh sh;

  cluster_arrive_relaxed();  // matched by the wait before the first remote store
  // Programmatic dependent launch: the next grid of the stream may place its
  // blocks as SMs free up; they wait (griddepcontrol.wait below) until this
  // grid has finished and its writes are visible.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const Layout L = make_layout(smem, pl);
  constexpr int es = (int)sizeof(T);
  const uint8_t *rowp = static_cast<const uint8_t *>(p.logits) + (int64_t)row * p.ld * es;

  // ---- slice geometry (a slice past the end of a short row is empty)
  const int64_t c0 = min((int64_t)rank * pl.slice, (int64_t)p.V);
  const int64_t c1 = min((int64_t)p.V, c0 + pl.slice);
  const uintptr_t a_c0 = reinterpret_cast<uintptr_t>(rowp + c0 * es);
  const uintptr_t a_c1 = reinterpret_cast<uintptr_t>(rowp + c1 * es);
  const uintptr_t a_al = a_c0 & ~(uintptr_t)15;
  const int64_t c0al = c0 - (int64_t)((a_c0 - a_al) / es);
  const uintptr_t b0 = (a_c0 + 15) & ~(uintptr_t)15;
  const uintptr_t b1 = a_c1 & ~(uintptr_t)15;
  const int64_t nbulk = (b1 > b0) ? (int64_t)(b1 - b0) : 0;
  const int hv = (int)((b0 - a_al) / 16);           // head fringe vectors (0 or 1)
  const int nbv = (int)(nbulk / 16);                // bulk vectors
  const int nvec = (int)((a_c1 - a_al + 15) / 16);  // all vectors of the slice
  const int nchunk = (int)((nbulk + CHUNK_BYTES - 1) / CHUNK_BYTES);
  uint4 *data4 = reinterpret_cast<uint4 *>(L.data);

  // no global memory is read before the previous grid of the stream (which
  // may have written the logits or the per-slot state) has completed
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- loads.  The small per-row inputs are loaded and staged first; the
  // slice follows as bulk copies of 64 KB chunks (one mbarrier each, all
  // issued by thread 0) once they are staged.  Requested behind the slice,
  // the small loads wait in the same memory queues as every row's stream
  // (measured: staged at ~3.3 us instead of ~1.9 us), and the setup that
  // needs them would wait with them.  A slice whose aligned interior maps
  // onto NVR vectors per thread keeps each vector's maximum in registers.
  const bool rt = nbv <= NT * NVR;  // uniform
  const bool has_hist = p.hist_ids && p.hist_len;
  // slot_idx costs one round trip before anything that depends on the slot
  const int slot = p.slot_idx ? p.slot_idx[row] : row;
  if (slot < 0) {  // padding row (uniform across the cluster): no load issued; write the padding outputs
    if (tid == 0 && rank == 0) {
      if (MODE == 0) {
        if (p.out_ids) p.out_ids[row] = p.vocab_offset;
        if (p.out_ids32) p.out_ids32[row] = (int32_t)p.vocab_offset;
        if (p.out_status) p.out_status[row] = 0;
      } else {
        uint32_t *rec = tp_send + (int64_t)row * pl.rec_words;
        rec[0] = __float_as_uint(-INFINITY);
        rec[1] = 0;
        rec[2] = 0;
        rec[3] = 0;
      }
    }
    if (MODE == 0 && (p.out_x || p.out_kept || p.out_probs)) {
      for (int64_t i = c0 + tid; i < c1; i += NT) {
        const int64_t o = (int64_t)row * p.V + i;
        if (p.out_x) p.out_x[o] = -INFINITY;
        if (p.out_kept) p.out_kept[o] = 0;
        if (p.out_probs) p.out_probs[o] = 0.0f;
      }
    }
    return;
  }
  // ---- the small loads first, into registers, so they are not queued
  // behind the slice: history length and words, the row's parameter words
  // (one per thread of warp 2), its uniform or Philox key and counter, the
  // fringe elements (warp 0) and the bias entries
  constexpr int HP = 2;  // history words prefetched per thread
  static_assert(HP == 2, "the insertion loop reads hpre[0] / hpre[1]");
  int hpre[HP] = {-1, -1};
  const int hlen = has_hist ? min(p.hist_len[slot], p.H) : 0;
  if (has_hist) {
    const int32_t *h = p.hist_ids + (int64_t)slot * p.H;
#pragma unroll
    for (int u = 0; u < HP; ++u) {
      const int j = u * NT + tid;
      hpre[u] = j < p.H ? h[j] : -1;
    }
  }
  uint64_t pword = 0;
  if (tid >= 64 && tid < 64 + NPARAM) {
    pword = param_word(p, tid - 64, slot);
  } else if (MODE == 0 && tid == 64 + NPARAM) {
    pword = p.uniforms ? (uint64_t)__float_as_uint(p.uniforms[row]) : (p.seed ? p.seed[slot] : 0ull);
  } else if (MODE == 0 && tid == 65 + NPARAM) {
    pword = (!p.uniforms && p.offset) ? p.offset[slot] : 0ull;
  }
  const int nfr = nvec - nbv;  // fringe vectors (at most one at each end)
  uint32_t fbits = Elem<T>::neg_inf();
  const bool has_fe = tid < nfr * VEC;  // this thread stages one fringe element
  int64_t fe = 0;  // its row position (may lie before the row: -inf there)
  if (has_fe) {
    const int f = tid / VEC;
    fe = c0al + (int64_t)(f < hv ? f : nbv + f) * VEC + tid % VEC;
    if (fe >= c0 && fe < c1) fbits = Elem<T>::load_bits(rowp, fe);
  }
  const bool bias_smem = p.bias_ids && p.NB <= BIAS_SMEM;
  int32_t bid = -1;
  float bval = 0.0f;
  if (bias_smem && tid < p.NB) {
    bid = p.bias_ids[(int64_t)slot * p.NB + tid];
    bval = p.bias_vals[(int64_t)slot * p.NB + tid];
  }
  // ---- the slice's chunk barriers (the copies start after the staging)
  if (tid == 0) {
    for (int j = 0; j < nchunk; ++j) mbar_init(&sh.mbar[j], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // ---- staging of the small values in shared memory
  if (tid >= 64 && tid < 64 + NPARAM) sh.pw[tid - 64] = (uint32_t)pword;
  else if (MODE == 0 && tid >= 64 + NPARAM && tid < 66 + NPARAM) sh.rng[tid - 64 - NPARAM] = pword;
  if (has_fe) {
    const int64_t pos = fe - c0al;
    if (es == 2) reinterpret_cast<uint16_t *>(L.data)[pos] = (uint16_t)fbits;
    else reinterpret_cast<uint32_t *>(L.data)[pos] = fbits;
  }
  if (bias_smem && tid < p.NB) {
    L.bias_id[tid] = bid;
    L.bias_val[tid] = bval;
  }
  if (tid == 0) {
    sh.nloc = 0;
    sh.scanned = 0;
    sh.status = 0;
    sh.n_spec = 0;
    sh.ht_fail = 0;
    sh.tp_ovf = 0;
    sh.pseudo = 0;
    sh.dumpx = 0;
    sh.nemit = 0;
    sh.cmax = okey(-INFINITY);
    sh.best = 0xFFFFFFFFu;
    sh.vcount = 0;
    tail_reset(sh);
  }

  const int64_t gbase = p.vocab_offset;
  const int64_t pos0_gid = gbase + c0al;  // gid of data position 0
  const bool has_spec = has_hist || p.seen_bits || p.bias_ids;

  // ---- setup while the logits are on their way: the skip bitmap
  // (disallowed and special positions; positions outside the slice are -inf
  // in the data) and the specials' hash table
  const int map_words = pl.map_bytes / 4;
  uint32_t *skip32 = reinterpret_cast<uint32_t *>(L.skip);
  if (has_spec)
    for (int i = tid; i < pl.ht_cap; i += NT) L.ht[i] = make_int2(-1, 0);
  for (int i = tid; i < NBIN; i += NT) L.queue[i] = 0;  // the top_k pre-cut's histogram
  if (p.allowed_bits || p.seen_bits) {
    // word by word: disallowed positions, and (seen-bit mode) the seen ones,
    // which also go into the seen map unless disallowed
    const uint32_t *aw = p.allowed_bits ? p.allowed_bits + (int64_t)slot * p.allowed_words : nullptr;
    const uint32_t *sw = p.seen_bits ? p.seen_bits + (int64_t)slot * p.seen_words : nullptr;
    for (int wi = tid; wi < map_words; wi += NT) {
      const int64_t e0 = c0al + (int64_t)wi * 32;
      const int64_t lo_in = min((int64_t)32, max((int64_t)0, c0 - e0));
      const int64_t hi_in = min((int64_t)32, max((int64_t)0, c1 - e0));
      uint32_t dis = 0u, sn = 0u;
      if (hi_in > lo_in) {
        const uint32_t hm = hi_in == 32 ? ~0u : ((1u << hi_in) - 1u);
        const uint32_t lm = lo_in == 32 ? ~0u : ((1u << lo_in) - 1u);
        const uint32_t inmask = hm & ~lm;
        if (aw) dis = inmask & ~(allowed32(aw, p.allowed_words, gbase + e0 + lo_in) << lo_in);
        if (sw) sn = inmask & ~dis & (allowed32(sw, p.seen_words, gbase + e0 + lo_in) << lo_in);
      }
      skip32[wi] = dis | sn;
      if (L.seen) L.seen[wi] = sn;
    }
  } else {
    uint4 *s4 = reinterpret_cast<uint4 *>(L.skip);
    for (int i = tid; i < map_words / 4; i += NT) s4[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();  // skip words written, table cleared, small values staged
  if (tid == 0) {  // the slice, chunk by chunk
    // (testing: with MSTAR_FLAG_TEST_WITHHOLD the last copy is never issued
    // and its barrier never completes, so its waits run out)
    const int nissue = (p.flags & MSTAR_FLAG_TEST_WITHHOLD) ? nchunk - 1 : nchunk;
    for (int j = 0; j < nissue; ++j) {
      const uint32_t bytes = (uint32_t)min((int64_t)CHUNK_BYTES, nbulk - (int64_t)j * CHUNK_BYTES);
      mbar_expect_tx(&sh.mbar[j], bytes);
      bulk_g2s(L.data + (b0 - a_al) + (int64_t)j * CHUNK_BYTES,
               reinterpret_cast<const void *>(b0 + (uintptr_t)j * CHUNK_BYTES), bytes, &sh.mbar[j]);
    }
  }
  if (tid == 64) {
    row_init(sh.row, sh.pw, p, row, p.V);
    // two-round TP: a row without top_k (or with one above the record's
    // capacity) leaves its shard values for the second round and, when the
    // shard has more ids than a record holds, sends the first tp_cap members
    // of its shard A set, marked as possibly partial
    if (MODE == 1 && pl.xdump && !sh.row.greedy && (!sh.row.topk || sh.row.K > pl.tp_cap)) {
      sh.dumpx = 1;
      if ((int64_t)pl.tp_cap < p.V) {
        sh.row.topk = true;
        sh.row.K = pl.tp_cap;
        sh.pseudo = 1;
      }
    }
  } else if (MODE == 0 && tid == 32) {
    sh.u = p.uniforms ? __uint_as_float((uint32_t)sh.rng[0]) : philox_uniform(sh.rng[0], sh.rng[1]);
  }
  // Specials: history ids and bias ids that fall in [c0, c1) (seen-mask
  // ids are in the seen map).  Each gets a skip bit (the max pass leaves it
  // out), a hash-table entry (its count and flags) and a list entry; its
  // final value is computed from the resident data after the max pass.  The
  // thread that creates a table entry sets the position's skip bit and
  // learns from the old bit whether the mask disallows the position.  The
  // table is complete before the logits are read.
  uint32_t *spec32 = reinterpret_cast<uint32_t *>(L.spec);
  auto new_entry = [&](int h) {  // list entry of a created table entry
    cg::coalesced_group g = cg::coalesced_threads();
    uint32_t cb = 0;
    if (g.thread_rank() == 0) cb = atomicAdd(&sh.n_spec, (uint32_t)g.size());
    const uint32_t ci = g.shfl(cb, 0) + g.thread_rank();
    if ((int)ci < pl.spec_cap) spec32[2 * ci] = (uint32_t)h;
    else sh.ht_fail = 1;
  };
  auto add_special = [&](int64_t e, int cnt) {
    int h;
    const int created = ht_insert(L.ht, pl.ht_cap, (int)e, cnt, h);
    if (created < 0) {
      sh.ht_fail = 1;
    } else if (created) {
      const int64_t pos = e - c0al;
      const uint32_t bit = 1u << (pos & 31);
      // seen-bit mode: a bias id that is also seen takes its count (1) here
      // and leaves the seen map, so it is visited once, from the list
      bool seen_here = false;
      if (L.seen) {
        seen_here = (atomicAnd(&L.seen[pos >> 5], ~bit) & bit) != 0u;
        if (seen_here) atomicAdd(&L.ht[h].y, 1);
      }
      // an already set skip bit of a position that is not seen means the
      // mask disallows it (seen positions in the map are allowed)
      if ((atomicOr(&skip32[pos >> 5], bit) & bit) && !seen_here) atomicOr(&L.ht[h].y, HT_MASKED);
      new_entry(h);
    }
  };
  // fn(e, count) for every materialized special occurrence of this slice
  // (e = position in the row): history ids and bias ids.  Seen-mask ids
  // are in the seen map (and the skip bitmap) already.
  auto for_each_special = [&](auto &&fn) {
    if (has_hist) {
#pragma unroll
      for (int u = 0; u < HP; ++u) {
        const int64_t g = (int64_t)hpre[u] - gbase;
        if (u * NT + tid < hlen && g >= c0 && g < c1) fn(g, 1);
      }
      const int32_t *h = p.hist_ids + (int64_t)slot * p.H;
      for (int j = HP * NT + tid; j < hlen; j += NT) {
        const int64_t g = (int64_t)h[j] - gbase;
        if (g >= c0 && g < c1) fn(g, 1);
      }
    }
    if (p.bias_ids && p.bias_vals) {
      const int32_t *bi = p.bias_ids + (int64_t)slot * p.NB;
      for (int j = tid; j < p.NB; j += NT) {
        const int32_t g = bi[j];
        if (g < 0) continue;
        const int64_t e = (int64_t)g - gbase;
        if (e >= c0 && e < c1) fn(e, 0);
      }
    }
  };
  if (has_spec) for_each_special(add_special);
  __syncthreads();  // bitmap, table and special list entries complete; row parameters in
  const Row r = sh.row;
  const Slice sl{data4, L.skip, nvec, pos0_gid, L.seen, map_words, rowp, c0al};
  const bool one = r.greedy || r.K == 1;

  // ---- max pass: the masked raw max of the slice (specials and disallowed
  // positions left out), then the specials' final values.  A slice of at
  // most NVR vectors per thread keeps each vector's raw max in registers for
  // the candidate pass; the slice stays resident in shared memory for the
  // later passes.
  Acc racc = Elem<T>::acc_init();
  float spec_max = -INFINITY;
  bool timed_out = false;
  Acc gm[NVR];
  const float penR = r.R, penF = r.F, penP = r.Pp;
  // Specials: bias (list order) -> penalties -> mask -> transform, after the
  // last block, from the resident data.  Entry i of the list holds its table
  // slot and becomes (x, id) in place.
  auto finalize = [&](int t0, int stride) {  // entries t0, t0 + stride, ...
    const bool bias_smem = p.bias_ids && p.NB <= BIAS_SMEM;
    const int32_t *bi = p.bias_ids ? p.bias_ids + (int64_t)slot * p.NB : nullptr;
    const float *bv = p.bias_vals ? p.bias_vals + (int64_t)slot * p.NB : nullptr;
    const int n = min((int)sh.n_spec, pl.spec_cap);
    const uint32_t *spec32 = reinterpret_cast<const uint32_t *>(L.spec);
    for (int i = t0; i < n; i += stride) {
      const int2 ent = L.ht[spec32[2 * i]];
      const int cnt = ent.y & ~HT_MASKED;
      float v = Elem<T>::smem_elem(L.data, ent.x - c0al);
      if (bi) {
        const int32_t gid = (int32_t)(ent.x + gbase);
        for (int j = 0; j < p.NB; ++j) {
          const int32_t id = bias_smem ? L.bias_id[j] : bi[j];
          if (id == gid) v = __fadd_rn(v, bias_smem ? L.bias_val[j] : bv[j]);
        }
      }
      if (cnt > 0) {
        v = (v > 0.0f) ? __fdiv_rn(v, penR) : __fmul_rn(v, penR);
        v = __fsub_rn(v, __fmul_rn(penF, (float)cnt));
        v = __fsub_rn(v, penP);
      }
      float x;
      if (v != v) x = v;
      else if (ent.y & HT_MASKED) x = -INFINITY;
      else x = xform(r, v);
      L.spec[i] = Cand{x, (uint32_t)(ent.x + gbase)};
      spec_max = fmaxf(spec_max, x);
    }
    for_each_seen<T>(sl, r, false, t0, stride, [&](const Cand &c, bool valid) {
      if (valid) spec_max = fmaxf(spec_max, c.x);
    });
  };
  uint32_t taint = 0;  // the thread's vectors (of gm) holding a skipped position
  if (rt) {
    // each vector's raw max (a few instructions) as its chunk lands, kept in
    // registers for the candidate pass; vectors with a skipped position
    // (special or disallowed; rare without an allowed mask) are then reduced
    // again, masked, and always rescanned by the candidate pass.  Row i of
    // the thread's vectors (NT consecutive vectors) lies in chunk i * NT * 16
    // / CHUNK_BYTES.
    static_assert(CHUNK_BYTES % (NT * 16) == 0, "a row of vectors lies in one chunk");
    constexpr int RPC = CHUNK_BYTES / (NT * 16);  // rows of vectors per chunk
#pragma unroll
    for (int i = 0; i < NVR; ++i) {
      const int q = i * NT + tid;
      if (q < nbv && Elem<T>::bits_of(L.skip, hv + q)) taint |= 1u << i;
    }
#pragma unroll
    for (int i = 0; i < NVR; ++i) {
      const int q = i * NT + tid;
      if (i % RPC == 0 && i / RPC < nchunk && !mbar_wait(&sh.mbar[i / RPC], 0)) timed_out = true;
      gm[i] = Elem<T>::acc_init();
      if (q < nbv) {
        gm[i] = Elem<T>::vred(data4[hv + q]);
        if (!((taint >> i) & 1u)) racc = Elem<T>::acc_max(racc, gm[i]);
      }
    }
    if (p.allowed_bits) {
      // an allowed mask taints nearly every vector: keep each tainted
      // vector's masked max, so the candidate pass rescans only vectors
      // whose allowed values reach the cut
      if (taint) {
#pragma unroll
        for (int i = 0; i < NVR; ++i)
          if ((taint >> i) & 1u) {
            gm[i] = Elem<T>::vred(load_masked<T>(sl, hv + i * NT + tid));
            racc = Elem<T>::acc_max(racc, gm[i]);
          }
      }
    } else {
      for (uint32_t t = taint; t; t &= t - 1u)
        racc = Elem<T>::acc_max(racc, Elem<T>::vred(load_masked<T>(sl, hv + (__ffs(t) - 1) * NT + tid)));
    }
  } else {
    constexpr int CV = CHUNK_BYTES / 16;
    for (int j = 0; j < nchunk; ++j) {
      if (!mbar_wait(&sh.mbar[j], 0)) timed_out = true;
      const int ke = hv + min(nbv, (j + 1) * CV);
      for (int k = hv + j * CV + tid; k < ke; k += NT)
        racc = Elem<T>::acc_max(racc, Elem<T>::vred(load_masked<T>(sl, k)));
    }
  }
  // the fringe vectors (at most one at each end, resident since the setup)
  for (int f = tid; f < nfr; f += NT)
    racc = Elem<T>::acc_max(racc, Elem<T>::vred(load_masked<T>(sl, f < hv ? f : nbv + f)));
  if (timed_out) atomicOr(&sh.status, MSTAR_STATUS_TIMEOUT);
  {  // this CTA's max over its non-special values
    float cmx = xform(r, Elem<T>::acc_f(racc));
    for (int o = 16; o; o >>= 1) cmx = fmaxf(cmx, __shfl_xor_sync(~0u, cmx, o));
    if (lane == 0 && cmx > -INFINITY) atomicMax(&sh.cmax, okey(cmx));
  }
  __syncthreads();  // non-special max complete; the slice is resident
  // ---- this CTA's value threshold theta(cm), cm its max: every member of
  // the row's A set (whose max m >= cm) has x >= theta(cm).  Warp 0 computes
  // it from the non-special max while the other warps finalize the specials;
  // it is redone only when a special holds the CTA max.
  const float cm_ns = okey_inv(sh.cmax);
  if (rt && r.topk && !one && (int)r.K <= TAIL_CAP / S) {
    // the top_k pre-cut's trigger: the untainted vectors within the usual
    // threshold span of the non-special max (an estimate: the cut itself is
    // taken against the exact theta)
    const float ta = fmaxf(__fsub_rn(cm_ns, 23.5f), r.minp ? __fadd_rn(cm_ns, __fsub_rn(r.lnMp, 0.01f)) : -INFINITY);
    uint32_t c = 0;
#pragma unroll
    for (int i = 0; i < NVR; ++i)
      c += (i * NT + tid < nbv && !((taint >> i) & 1u) && xform(r, Elem<T>::acc_f(gm[i])) >= ta) ? 1u : 0u;
    c = __reduce_add_sync(~0u, c);
    if (lane == 0 && c) atomicAdd(&sh.vcount, c);
  }
  if (tid < 32) {
    const float t = cm_ns > -INFINITY ? choose_theta(r, cm_ns) : INFINITY;
    if (lane == 0) sh.theta = t;
  } else if (has_spec) {
    finalize(tid - 32, NT - 32);
    float smx = spec_max;
    for (int o = 16; o; o >>= 1) smx = fmaxf(smx, __shfl_xor_sync(~0u, smx, o));
    if (lane == 0 && smx > -INFINITY) atomicMax(&sh.cmax, okey(smx));
  }
  __syncthreads();  // specials final, CTA max complete
  const float cm = okey_inv(sh.cmax);  // this CTA's max (transformed)
  if (cm != cm_ns) {  // uniform: a special holds the CTA max
    if (tid < 32) {
      const float t = choose_theta(r, cm);
      if (lane == 0) sh.theta = t;
    }
    __syncthreads();
  }
  const int nspec = min((int)sh.n_spec, pl.spec_cap);
  if (MODE == 1 && pl.xdump && sh.dumpx) {  // uniform: the shard values for the second round
    RowCtx dc;
    dc.p = &p;
    dc.L = L;
    dc.sl = sl;
    dc.r = r;
    dc.rowp = rowp;
    dc.nspec = nspec;
    dc.row = row;
    dc.slot = slot;
    dc.c0 = c0;
    dc.c1 = c1;
    dc.gbase = gbase;
    float *xo = pl.xdump + (int64_t)row * p.V;
    dense_values<T>(dc, [&](int64_t e, float x) { xo[e] = x; });
  }
  const float theta_l = sh.theta;
  const int capq = TAIL_CAP / S;  // candidates each CTA may push to the leader
  cluster_wait();                 // every CTA of the cluster runs: remote stores are safe

  // ---- cluster-wide top_k cut, for a top_k row whose K exceeds what one CTA
  // may push (its K largest could then not be cut CTA by CTA): the CTAs
  // exchange their maxima, add histograms of their untainted vector maxima
  // and their specials' values over common value bins [theta(m), m] into the
  // leader's shared memory, and each reads the first bin from the top where
  // the count reaches K.  K items (distinct values of the row) lie above that
  // bin's lower edge, so no value at or below it is among the row's K
  // largest.  Two cluster barriers instead of the general path's rounds;
  // taken by every CTA of the cluster or by none (it depends on the row's
  // parameters and the plan only).
  bool gk = false;
  float gk_x = -INFINITY;
  if (MODE == 0 && !one && r.topk && r.K > capq && r.K <= GCUT_MAX_K &&
      pl.slice * es <= (int64_t)NT * NVR * 16) {  // cluster-uniform; every CTA keeps its maxima in registers
    if (tid < S) cluster.map_shared_rank(&sh, tid)->maxes[rank] = cm;
    cluster.sync();  // maxima delivered; every histogram cleared in the setup
    float mq = lane < S ? sh.maxes[lane] : -INFINITY;
    for (int o = 16; o; o >>= 1) mq = fmaxf(mq, __shfl_xor_sync(~0u, mq, o));
    const float mg = mq;  // the row max
    const float tg = mg > -INFINITY ? choose_theta(r, mg) : INFINITY;  // every warp: same value
    VBins vb;
    vb.m = mg;
    vb.w = __fmul_rn(__fsub_rn(mg, tg), 1.0f / NBIN);
    vb.iw = 1.0f / vb.w;
    const bool ok = mg > -INFINITY && vb.w > 0.0f && vb.w < INFINITY && vb.iw < INFINITY;  // cluster-uniform
    uint32_t *lhist = cluster.map_shared_rank(reinterpret_cast<uint32_t *>(L.queue), 0);
    if (ok) {
#pragma unroll
      for (int i = 0; i < NVR; ++i) {
        const float gx = xform(r, Elem<T>::acc_f(gm[i]));
        if (i * NT + tid < nbv && !((taint >> i) & 1u) && gx >= tg) atomicAdd(&lhist[vb_bin(vb, gx)], 1u);
      }
      for (int i = tid; i < nspec; i += NT) {
        const float x = L.spec[i].x;
        if (x >= tg) atomicAdd(&lhist[vb_bin(vb, x)], 1u);
      }
    }
    cluster.sync();  // the leader's histogram complete
    if (ok) {
      if (tid < 32) {
        const int bk = vb_kbin(lhist, (uint32_t)r.K);
        if (lane == 0) sh.kcut_bin = bk;
      }
      __syncthreads();
      if (sh.kcut_bin < NBIN - 1) {
        gk = true;
        gk_x = vb_edge(vb, sh.kcut_bin + 1);
      }
    }
  }

  // ---- candidates: x >= theta(cm) (or x == cm for greedy / top-1),
  // pushed into the leader's region: the vectors whose max (kept in registers)
  // reaches the cut (a bulk-copied slice: every vector), the fringe vectors
  // and the specials.  Once this CTA holds more candidates than it may push
  // the scan stops and the row takes the general path (which scans again) --
  // unless it is a top_k row: the row's K largest are among every CTA's own
  // K largest, so the push is redone leaving out what lies below the value
  // bin holding this CTA's K-th largest candidate (bin b holds
  // E(b+1) < x <= E(b), E(b) = cm - b w, w = (cm - theta) / NBIN), found by
  // one histogram pass over the resident slice and the specials.  Ties at
  // the cut are all pushed.
  if (cm > -INFINITY) {
    const float tcut = one ? cm : theta_l;
    Cand *const lead = cluster.map_shared_rank(L.lcand, 0) + rank * capq;
    uint32_t best = 0xFFFFFFFFu;
    bool kcut = gk;
    float kcut_x = gk_x;  // pushed: x > kcut_x (with kcut)
    // one vector per lane per step (warp-uniform step count); the passing
    // values are appended with one atomic per warp
    auto scan_vec = [&](int k, bool valid) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      bool any = false;
      if (valid) {
        v = load_masked<T>(sl, k);
        any = xform(r, Elem<T>::vmax(v)) >= tcut;
      }
      const uint32_t gid0 = (uint32_t)(pos0_gid + (int64_t)k * VEC);
      uint32_t pm = 0;
      if (any) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float x = xform(r, Elem<T>::get(v, j));
          if (one) {
            if (x == cm) best = min(best, gid0 + (uint32_t)j);
          } else if (x >= theta_l && (!kcut || x > kcut_x)) {
            pm |= 1u << j;
          }
        }
      }
      if (one || !__any_sync(~0u, pm != 0u)) return;
      uint32_t o = warp_reserve(&sh.nloc, (uint32_t)__popc(pm));
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        if (!((pm >> j) & 1u)) continue;
        if (o < (uint32_t)capq) lead[o] = Cand{xform(r, Elem<T>::get(v, j)), gid0 + (uint32_t)j};
        ++o;
      }
    };
    auto push_special = [&](const Cand &c, bool valid) {  // all 32 lanes
      if (one) {
        if (valid && c.x == cm) best = min(best, c.gid);
        return;
      }
      const bool pass = valid && c.x >= theta_l && (!kcut || c.x > kcut_x);
      if (!__any_sync(~0u, pass)) return;
      const uint32_t o = warp_reserve(&sh.nloc, pass ? 1u : 0u);
      if (pass && o < (uint32_t)capq) lead[o] = c;
    };
    // (one vector per lane per step, warp-uniform step counts)
    auto push_all = [&]() {
      int stop = -1;  // warp-uniform: the step at which this warp stopped
      auto held_over = [&]() {
        return __shfl_sync(~0u, *reinterpret_cast<volatile uint32_t *>(&sh.nloc), 0) > (uint32_t)capq;
      };
      if (rt) {
        // the thread's vectors whose max reaches the cut, as a bit mask (one
        // compact unrolled test), then one rolled loop over the set bits:
        // the scan's code is instantiated once, not once per vector
        // (a tainted vector's kept max is its raw max, which bounds its
        // masked max, or with an allowed mask the masked max itself)
        uint32_t pm = 0;
#pragma unroll
        for (int i = 0; i < NVR; ++i) {
          const float gx = xform(r, Elem<T>::acc_f(gm[i]));
          pm |= (i * NT + tid < nbv && gx >= tcut && (!kcut || gx > kcut_x)) ? 1u << i : 0u;
        }
        int steps = 0;
        while (__any_sync(~0u, pm != 0u)) {  // warp-uniform
          if (held_over()) {
            stop = steps;
            break;
          }
          const bool valid = pm != 0u;
          const int i = valid ? __ffs(pm) - 1 : 0;
          pm &= pm - 1u;
          scan_vec(hv + i * NT + tid, valid);
          ++steps;
        }
        if (stop >= 0 && lane == 0) atomicAdd(&sh.scanned, (uint32_t)stop * 32u + 1u);
      } else {
        int k0 = 0;
        for (; k0 < nbv; k0 += NT) {
          if (held_over()) break;
          scan_vec(hv + k0 + tid, k0 + tid < nbv);
        }
        if (k0 < nbv && lane == 0) atomicAdd(&sh.scanned, (uint32_t)k0 / NWARP + 1u);
      }
      if (tid < 32) scan_vec(lane < hv ? lane : nbv + lane, lane < nfr);  // the fringe vectors
      for (int i0 = 0; i0 < nspec; i0 += NT) {
        const int i = i0 + tid;
        const bool valid = i < nspec;
        push_special(valid ? L.spec[i] : Cand{-INFINITY, 0u}, valid);
      }
      for_each_seen<T>(sl, r, false, tid, NT, push_special);
    };
    // Pre-cut of a top_k row from the vector maxima kept in registers: if at
    // least K untainted vectors have a max in value bins 0..b, this CTA's K-th
    // largest value is > E(b + 1), so nothing at or below E(b + 1) is among
    // its K largest (nor the row's).  Taken when the vectors reaching theta
    // are many times K; it keeps the push and the leader's sort near K
    // candidates per CTA instead of every value above theta.
    if (rt && !one && r.topk && r.K <= capq && sh.vcount > (uint32_t)(PRECUT_FACTOR * r.K)) {  // CTA-uniform
      uint32_t pv = 0;  // untainted vectors reaching theta
#pragma unroll
      for (int i = 0; i < NVR; ++i)
        pv |= (i * NT + tid < nbv && !((taint >> i) & 1u) && xform(r, Elem<T>::acc_f(gm[i])) >= theta_l) ? 1u << i
                                                                                                           : 0u;
      VBins vb;
      vb.m = cm;
      vb.w = __fmul_rn(__fsub_rn(cm, theta_l), 1.0f / NBIN);
      vb.iw = 1.0f / vb.w;
      if (vb.w > 0.0f && vb.w < INFINITY && vb.iw < INFINITY) {  // CTA-uniform
        uint32_t *hist = reinterpret_cast<uint32_t *>(L.queue);  // cleared in the setup
        for (uint32_t t = pv; t; t &= t - 1u) {
          const int k = hv + (__ffs(t) - 1) * NT + tid;
          atomicAdd(&hist[vb_bin(vb, xform(r, Elem<T>::vmax(data4[k])))], 1u);
        }
        __syncthreads();
        if (tid < 32) {
          const int bk = vb_kbin(hist, (uint32_t)r.K);
          if (lane == 0) sh.kcut_bin = bk;
        }
        __syncthreads();
        const int bk = sh.kcut_bin;
        if (bk < NBIN - 1) {
          kcut = true;
          kcut_x = vb_edge(vb, bk + 1);
        }
      }
    }
    push_all();
    __syncthreads();
    if (!kcut && !one && r.topk && r.K <= capq && sh.nloc > (uint32_t)capq) {  // CTA-uniform: a top_k row overflowed
      VBins vb;
      vb.m = cm;
      vb.w = __fmul_rn(__fsub_rn(cm, theta_l), 1.0f / NBIN);
      vb.iw = 1.0f / vb.w;
      if (vb.w > 0.0f && vb.w < INFINITY && vb.iw < INFINITY) {  // CTA-uniform
        uint32_t *hist = reinterpret_cast<uint32_t *>(L.queue);
        for (int i = tid; i < NBIN; i += NT) hist[i] = 0u;
        __syncthreads();
        for (int k = tid; k < nvec; k += NT) {
          const uint4 v = load_masked<T>(sl, k);
          if (!(xform(r, Elem<T>::vmax(v)) >= theta_l)) continue;
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            const float x = xform(r, Elem<T>::get(v, j));
            if (x >= theta_l) atomicAdd(&hist[vb_bin(vb, x)], 1u);
          }
        }
        for (int i = tid; i < nspec; i += NT) {
          const float x = L.spec[i].x;
          if (x >= theta_l) atomicAdd(&hist[vb_bin(vb, x)], 1u);
        }
        for_each_seen<T>(sl, r, false, tid, NT, [&](const Cand &c, bool valid) {
          if (valid && c.x >= theta_l) atomicAdd(&hist[vb_bin(vb, c.x)], 1u);
        });
        __syncthreads();
        if (tid < 32) {  // the first bin where the count from the top reaches K
          const int bk = vb_kbin(hist, (uint32_t)r.K);
          if (lane == 0) sh.kcut_bin = bk;
        }
        __syncthreads();
        const int bk = sh.kcut_bin;
        if (bk < NBIN - 1) {
          kcut = true;
          kcut_x = vb_edge(vb, bk + 1);
        }
      }
      if (kcut) {  // CTA-uniform
        if (tid == 0) {
          sh.nloc = 0;
          sh.scanned = 0;
        }
        __syncthreads();
        push_all();
      }
    }
    if (best != 0xFFFFFFFFu) atomicMin(&sh.best, best);
  }
  __syncthreads();
  if (tid < S) {  // push this CTA's max, count, status and lowest id to every CTA
    CtaSh *peer = cluster.map_shared_rank(&sh, tid);
    peer->maxes[rank] = cm;
    peer->gcnt[rank] = sh.nloc;
    peer->gstat[rank] = sh.status | (sh.ht_fail ? (uint32_t)MSTAR_STATUS_SPECIAL_OVERFLOW : 0u);
    peer->gmin[rank] = sh.best;
  }
  cluster.sync();  // #1: candidates, maxima and counts delivered

  // every CTA takes the same decision from the delivered values
  const bool debug = MODE == 0 && (p.out_x || p.out_kept || p.out_probs);
  float m;
  bool fast;
  {
    float mq = lane < S ? sh.maxes[lane] : -INFINITY;
    for (int o = 16; o; o >>= 1) mq = fmaxf(mq, __shfl_xor_sync(~0u, mq, o));
    m = mq;
    const uint32_t cq = lane < S ? sh.gcnt[lane] : 0u;
    const bool ovf = __any_sync(~0u, cq > (uint32_t)capq);
    fast = !(m > -INFINITY) || one || (!ovf && !(p.flags & MSTAR_FLAG_FORCE_GENERAL));
  }
  const bool empty = !(m > -INFINITY);
  if (fast && rank != 0 && !debug) return;  // nothing of this CTA is read any more
  const uint32_t km = okey(m);
  if (tid < 32) {
    const uint32_t cq = lane < S ? min(sh.gcnt[lane], (uint32_t)capq) : 0u;
    uint32_t inc = cq;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(~0u, inc, o);
      if (lane >= o) inc += v;
    }
    const uint32_t st = __reduce_or_sync(~0u, lane < S ? sh.gstat[lane] : 0u);
    const uint32_t mg = __reduce_min_sync(~0u, (lane < S && sh.maxes[lane] == m) ? sh.gmin[lane] : 0xFFFFFFFFu);
    // the general path needs the row's own value threshold
    const float tg = (!fast && !empty) ? choose_theta(r, m) : INFINITY;
    if (lane < 16) sh.goff[lane] = inc - cq;
    if (lane == 31) sh.ncand = inc;
    if (lane == 0) {
      sh.theta = tg;
      sh.min_all = mg;
      sh.res.m = m;
      sh.res.theta = tg;
      sh.res.greedy = r.greedy;
      sh.res.empty = empty;
      sh.res.token = 0;
      sh.res.WK = 0;
      sh.res.ckK = 0;
      sh.res.status = st;
    }
  } else if (fast && rank == 0) {  // the leader's slice data is dead: clear the one-pass tail's counters
    tail_clear1(tail_scratch(L.data), tid - 32, NT - 32);
  }
  __syncthreads();
  const float theta = sh.theta;
  uint32_t *rec = MODE == 1 ? tp_send + (int64_t)row * pl.rec_words : nullptr;
  RowCtx ctx;
  if (!fast || debug) {
    ctx.p = &p;
    ctx.pl = &pl;
    ctx.L = L;
    ctx.sl = sl;
    ctx.r = r;
    ctx.rowp = rowp;
    ctx.m = m;
    ctx.theta = theta;
    ctx.u = MODE == 0 ? sh.u : 0.0f;
    ctx.km = km;
    ctx.nspec = nspec;
    ctx.rank = rank;
    ctx.S = S;
    ctx.row = row;
    ctx.slot = slot;
    ctx.c0 = c0;
    ctx.c1 = c1;
    ctx.gbase = gbase;
    ctx.rec = rec;
    ctx.empty = empty;
  }
  if (fast) {
    if (rank == 0 && !empty) {
      if (one) {
        if (tid == 0) {
          sh.res.token = sh.min_all;
          sh.res.WK = 4294967296ull;
          sh.res.ckK = (uint64_t)sh.min_all;
          sh.nemit = -1;
        }
      } else {
        // the S pushed candidate lists (list q at lcand + q * capq, its
        // entries numbered from goff[q] in the gathered order)
        const TailScr ts = tail_scratch(L.data);  // the leader's slice data is dead by now
        const int n = (int)sh.ncand;
        uint64_t kmn = ~0ull, kmx = 0ull;
        uint32_t np = 0;
        if (n > RANK_SMALL && n <= NT) {  // one candidate per thread, kept in registers
          const bool valid = tid < n;
          uint64_t key = 0, w = 0;
          if (valid) {
            int q = 0;
            while (q + 1 < S && tid >= (int)sh.goff[q + 1]) ++q;
            tail_put(r, m, km, L.lcand[q * capq + (tid - (int)sh.goff[q])], tid, ts, kmn, kmx, np);
            key = ts.K[tid];
            w = ts.W[tid];
          }
          tail_finish1<MODE>(r, MODE == 0 ? sh.u : 0.0f, km, n, valid, key, w, kmn, kmx, pl.tp_cap, rec, ts, sh);
        } else {
          for (int i = tid; i < n; i += NT) {  // one candidate per thread
            int q = 0;
            while (q + 1 < S && i >= (int)sh.goff[q + 1]) ++q;
            tail_put(r, m, km, L.lcand[q * capq + (i - (int)sh.goff[q])], i, ts, kmn, kmx, np);
          }
          tail_finish<MODE>(r, MODE == 0 ? sh.u : 0.0f, km, n, kmn, kmx, np, pl.tp_cap, rec, ts, sh);
        }
      }
    }
  } else {
    general_path<T, MODE>(ctx, sh);
  }

  // ---- leader: outputs and state updates
  if (rank == 0) {
    __syncthreads();
    if (MODE == 0) {
      if (tid == 0) {
        uint32_t status = sh.res.status;
        uint32_t token = sh.res.token;
        if (empty) {
          status |= MSTAR_STATUS_EMPTY;
          token = (uint32_t)gbase;
        }
        sh.res.status = status;
        write_row_outputs(p, row, slot, token, status);
      }
    } else {
      const int nemit = sh.nemit;
      const bool ovf = sh.tp_ovf || (nemit > pl.tp_cap);
      if (tid == 0) {
        rec[0] = __float_as_uint(empty ? -INFINITY : m);
        const uint32_t st =
            sh.res.status | (ovf ? MSTAR_STATUS_TP_OVERFLOW : 0u) | (empty ? MSTAR_STATUS_EMPTY : 0u);
        if (nemit < 0) {
          rec[1] = 1;
          rec[4] = __float_as_uint(m);
          rec[5] = sh.res.token;
        } else {
          rec[1] = ovf ? 0u : (uint32_t)nemit;
        }
        rec[2] = st;
        rec[3] = sh.pseudo ? 1u : 0u;  // bit 0: the record holds at most the first tp_cap members
      }
    }
  }
  if (debug) {
    cluster.sync();
    debug_dense<T>(ctx, sh);
  }
  if (!fast || debug) cluster.sync();  // keep shared memory alive until every remote access is done
}

// ------------------------------------------------------------ small rows

// Rows of at most SMALL_V ids (a codec vocabulary sampled over and over in
// the Talker's per-frame depth loop, python/mstar_rs/models/qwen3_omni.py:
// 1085-1094) take a kernel of their own: one CTA per row, the row in
// registers (SMALL_EPT ids per thread), occurrence counts in a dense
// shared-memory array instead of the hash table, every candidate (x >= the
// value threshold) gathered once and ordered by the large-row tail's bucket
// sort (pairwise ranking up to 256 candidates), then the same resolution.
// No cluster, no bulk copies, no general path: a handful of block-wide steps.
constexpr int SMALL_V = 4096;
constexpr int SMALL_EPT = SMALL_V / NT;  // ids per thread
// counts (later the tail's positions) | biased-id bitmap | keys, weights,
// ranked keys, ranked weights, prefixes | bucket counts, masses | bias list
constexpr int SMALL_OFF_BMARK = SMALL_V * 4;
constexpr int SMALL_OFF_K = SMALL_OFF_BMARK + SMALL_V / 8;
constexpr int SMALL_OFF_BC = SMALL_OFF_K + 5 * SMALL_V * 8;
constexpr int SMALL_OFF_BIAS = SMALL_OFF_BC + NBK * 12;
constexpr int SMALL_SMEM = SMALL_OFF_BIAS + BIAS_SMEM * 8;
static_assert(SMALL_V % NT == 0, "small rows: whole ids per thread");
static_assert(SMALL_V <= 65536 && NBK % NT == 0, "small rows: tail positions and bucket scan");

// Value-bucket sort of a small row's n <= SMALL_V gathered candidates:
// SMALL_NBUC buckets uniform in x over the A range below the row max (as
// tail_bucket_sort, eight times finer: a row of SMALL_V Gaussian values puts
// a handful in each), a counting pass, a block scan of the counts, a scatter
// into bucket order and a rank inside each bucket.  Leaves keys, weights and
// exclusive weight prefixes in rank order in K / W / RS (the gathered
// arrays are dead after the scatter; RK / RW hold the bucket order, RS the
// bucket counts and starts until the prefix pass).  Returns false, having
// sorted nothing, when a bucket of A holds more than BUCKET_MAX candidates
// (runs of exact ties).  Block-wide; ends with a barrier.
constexpr int SMALL_NBUC = 2048;
static_assert(SMALL_NBUC % NT == 0 && SMALL_NBUC * 8 <= SMALL_V * 8, "small rows: bucket scan and counts");
__device__ bool small_bucket_sort(const Row &r, uint32_t km, int n, const TailScr &s, CtaSh &sh) {
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const float m = okey_inv(km);
  const float span = fmaxf(r.minp ? fminf(23.5f, __fadd_rn(-r.lnMp, 0.25f)) : 23.5f, 1e-3f);
  const float sc = (float)SMALL_NBUC / span;
  constexpr uint32_t LAST = SMALL_NBUC - 1;  // x at or below m - span * LAST / NBUC: outside A
  auto bucket_of = [&](uint64_t key) {       // monotone in the key
    const float x = okey_inv(km - (uint32_t)(key >> 32));
    const float g = __fmul_rn(__fsub_rn(m, x), sc);
    return g >= (float)LAST ? LAST : (g > 0.0f ? (uint32_t)g : 0u);
  };
  uint32_t *cnt = reinterpret_cast<uint32_t *>(s.RS), *start = cnt + SMALL_NBUC;
  uint64_t *BK = s.RK, *BW = s.RW;
  for (int b = t; b < SMALL_NBUC; b += NT) cnt[b] = 0u;
  __syncthreads();
  for (int i = t; i < n; i += NT) {
    const uint32_t b = bucket_of(s.K[i]);
    s.P[i] = (b << 16) | atomicAdd(&cnt[b], 1u);
  }
  __syncthreads();
  constexpr int PER = SMALL_NBUC / NT;
  uint32_t c[PER], tot = 0, big = 0;
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    c[q] = cnt[t * PER + q];
    tot += c[q];
    big |= (t * PER + q < (int)LAST && c[q] > BUCKET_MAX) ? 1u : 0u;
  }
  uint32_t inc = tot;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(~0u, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) sh.red_u32[wid] = inc;
  if (__syncthreads_or((int)big)) return false;  // uniform
  uint32_t run = inc - tot;
  for (int w = 0; w < wid; ++w) run += sh.red_u32[w];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    start[t * PER + q] = run;
    run += c[q];
  }
  __syncthreads();
  // with top_k only the first K ranks are read: buckets starting at or past
  // rank K are neither placed nor ranked
  const uint32_t lim = r.topk ? (uint32_t)r.K : 0xFFFFFFFFu;
  for (int i = t; i < n; i += NT) {
    const uint32_t pb = s.P[i];
    if (start[pb >> 16] >= lim) continue;
    const uint32_t dst = start[pb >> 16] + (pb & 0xFFFFu);
    BK[dst] = s.K[i];
    BW[dst] = s.W[i];
  }
  __syncthreads();
  uint32_t placed = (uint32_t)n;
  if (lim < (uint32_t)n) {
    int lo = 0, hi = (int)LAST;  // the last bucket whose start is < lim (starts are non-decreasing)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (start[mid] < lim) lo = mid;
      else hi = mid - 1;
    }
    placed = start[lo] + cnt[lo];
  }
  for (int q = t; q < (int)placed; q += NT) {  // rank inside the bucket
    const uint64_t key = BK[q];
    const uint32_t b = bucket_of(key);
    const uint32_t st = start[b], en = st + cnt[b];
    uint32_t rk = (uint32_t)q - st;  // outside A: any order
    if (b < LAST) {
      rk = 0;
      for (uint32_t j = st; j < en; ++j) rk += BK[j] < key ? 1u : 0u;
    }
    s.K[st + rk] = key;
    s.W[st + rk] = BW[q];
  }
  __syncthreads();
  {  // exclusive prefix of the weights in rank order, a segment per thread
    const int seg = (int)((placed + NT - 1) / NT);
    const int a0 = min((int)placed, t * seg), a1 = min((int)placed, a0 + seg);
    uint64_t loc = 0;
    for (int j = a0; j < a1; ++j) loc += s.W[j];
    uint64_t tot64;
    uint64_t run64 = block_exscan_u64(loc, tot64, sh);
    for (int j = a0; j < a1; ++j) {
      s.RS[j] = run64;
      run64 += s.W[j];
    }
  }
  __syncthreads();
  return true;
}

template <typename T>
__global__ void __launch_bounds__(NT, 1) small_kernel(const mstar_sampler_params_t p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ CtaSh sh;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const int V = p.V;
  const int64_t gbase = p.vocab_offset;
  uint32_t *cnt = reinterpret_cast<uint32_t *>(smem);
  uint32_t *bmark = reinterpret_cast<uint32_t *>(smem + SMALL_OFF_BMARK);  // ids with a bias entry
  int32_t *bid = reinterpret_cast<int32_t *>(smem + SMALL_OFF_BIAS);
  float *bval = reinterpret_cast<float *>(bid + BIAS_SMEM);
  TailScr ts;
  ts.K = reinterpret_cast<uint64_t *>(smem + SMALL_OFF_K);
  ts.W = ts.K + SMALL_V;
  ts.RK = ts.W + SMALL_V;
  ts.RW = ts.RK + SMALL_V;
  ts.RS = ts.RW + SMALL_V;
  ts.P = cnt;  // the counts are dead once the transformed values are in registers
  ts.bc = reinterpret_cast<uint32_t *>(smem + SMALL_OFF_BC);
  ts.bm = reinterpret_cast<uint64_t *>(smem + SMALL_OFF_BC + NBK * 4);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int slot = p.slot_idx ? p.slot_idx[row] : row;
  const bool debug = p.out_x || p.out_kept || p.out_probs;
  if (slot < 0) {
    if (tid == 0) {
      if (p.out_ids) p.out_ids[row] = gbase;
      if (p.out_ids32) p.out_ids32[row] = (int32_t)gbase;
      if (p.out_status) p.out_status[row] = 0;
    }
    for (int i = tid; debug && i < V; i += NT) {
      const int64_t o = (int64_t)row * V + i;
      if (p.out_x) p.out_x[o] = -INFINITY;
      if (p.out_kept) p.out_kept[o] = 0;
      if (p.out_probs) p.out_probs[o] = 0.0f;
    }
    return;
  }
  // the row (id i = tid + NT * j), the parameters, the draw
  const uint8_t *rowp = static_cast<const uint8_t *>(p.logits) + (int64_t)row * p.ld * sizeof(T);
  float raw[SMALL_EPT];
#pragma unroll
  for (int j = 0; j < SMALL_EPT; ++j) {
    const int i = tid + NT * j;
    raw[j] = i < V ? Elem<T>::load(rowp, i) : -INFINITY;
  }
  if (tid == 0) {
    sh.n_spec = 0;
    sh.npass = 0;
    sh.cnt_k = 0;
    sh.best = 0xFFFFFFFFu;
    sh.cmax = okey(-INFINITY);
    sh.kmin = ~0ull;
    sh.kmax = 0ull;
    sh.res.token = 0;
    sh.res.WK = 0;
    sh.res.ckK = 0;
  } else if (tid == 64) {
    row_init(sh.row, p, row, slot, V);
  } else if (tid == 32) {
    sh.u = p.uniforms ? p.uniforms[row]
                      : philox_uniform(p.seed ? p.seed[slot] : 0ull, p.offset ? p.offset[slot] : 0ull);
  }
  for (int i = tid; i < SMALL_V; i += NT) cnt[i] = 0u;
  for (int i = tid; i < SMALL_V / 32; i += NT) bmark[i] = 0u;
  const bool bias = p.bias_ids && p.bias_vals;
  const bool bias_smem = bias && p.NB <= BIAS_SMEM;
  for (int j = tid; bias_smem && j < p.NB; j += NT) {
    bid[j] = p.bias_ids[(int64_t)slot * p.NB + j];
    bval[j] = p.bias_vals[(int64_t)slot * p.NB + j];
  }
  __syncthreads();
  // occurrence counts (history ring) and each biased id's first bias entry
  if (p.hist_ids && p.hist_len) {
    const int32_t *h = p.hist_ids + (int64_t)slot * p.H;
    const int hl = min(p.hist_len[slot], p.H);
    for (int j = tid; j < hl; j += NT) {
      const int64_t e = (int64_t)h[j] - gbase;
      if (e >= 0 && e < V) atomicAdd(&cnt[e], 1u);
    }
  }
  if (bias) {
    const int32_t *bi = p.bias_ids + (int64_t)slot * p.NB;
    for (int j = tid; j < p.NB; j += NT) {
      const int32_t id = bias_smem ? bid[j] : bi[j];
      const int64_t e = (int64_t)id - gbase;
      if (id >= 0 && e >= 0 && e < V) atomicOr(&bmark[e >> 5], 1u << (e & 31));
    }
  }
  __syncthreads();
  const Row r = sh.row;
  const uint32_t *sw = p.seen_bits ? p.seen_bits + (int64_t)slot * p.seen_words : nullptr;
  const uint32_t *aw = p.allowed_bits ? p.allowed_bits + (int64_t)slot * p.allowed_words : nullptr;
  float x[SMALL_EPT];
  float tmax = -INFINITY;
#pragma unroll
  for (int j = 0; j < SMALL_EPT; ++j) {
    const int i = tid + NT * j;
    float v = raw[j];
    x[j] = -INFINITY;
    if (i >= V) continue;
    const int64_t g = gbase + i;
    if (bias && ((bmark[i >> 5] >> (i & 31)) & 1u)) {
      const int32_t *bi = p.bias_ids + (int64_t)slot * p.NB;
      const float *bv = p.bias_vals + (int64_t)slot * p.NB;
      for (int q = 0; q < p.NB; ++q) {  // bias entries in list order
        const int32_t id = bias_smem ? bid[q] : bi[q];
        if (id == (int32_t)g) v = __fadd_rn(v, bias_smem ? bval[q] : bv[q]);
      }
    }
    const int c = sw ? (int)((sw[g >> 5] >> (g & 31)) & 1u) : (int)cnt[i];
    if (c > 0) {
      v = (v > 0.0f) ? __fdiv_rn(v, r.R) : __fmul_rn(v, r.R);
      v = __fsub_rn(v, __fmul_rn(r.F, (float)c));
      v = __fsub_rn(v, r.Pp);
    }
    const bool allowed = !aw || ((aw[g >> 5] >> (g & 31)) & 1u);
    if (v != v) x[j] = v;
    else if (!allowed) x[j] = -INFINITY;
    else x[j] = xform(r, v);
    tmax = fmaxf(tmax, x[j]);
  }
  // row max; greedy / top-1: the lowest id at the max
  for (int o = 16; o; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(~0u, tmax, o));
  if (lane == 0 && tmax > -INFINITY) atomicMax(&sh.cmax, okey(tmax));
  __syncthreads();
  const float m = okey_inv(sh.cmax);
  const bool empty = !(m > -INFINITY);
  const bool one = r.greedy || r.K == 1;
  uint32_t token = (uint32_t)gbase, status = 0;
  if (empty) {
    status = MSTAR_STATUS_EMPTY;
  } else if (one) {
    uint32_t best = 0xFFFFFFFFu;
#pragma unroll
    for (int j = 0; j < SMALL_EPT; ++j)
      if (x[j] == m) best = min(best, (uint32_t)(gbase + tid + NT * j));
    best = __reduce_min_sync(~0u, best);
    if (lane == 0) atomicMin(&sh.best, best);
    __syncthreads();
    token = sh.best;
    if (tid == 0) {
      sh.res.token = token;
      sh.res.WK = 4294967296ull;
      sh.res.ckK = (uint64_t)token;
    }
  } else {
    if (tid < 32) {
      const float t = choose_theta(r, m);
      if (lane == 0) sh.theta = t;
    }
    __syncthreads();
    const float theta = sh.theta;
    const uint32_t km = okey(m);
    // candidates (x >= theta): order keys and weights, compacted
    uint32_t mine = 0;
#pragma unroll
    for (int j = 0; j < SMALL_EPT; ++j) mine += (x[j] >= theta) ? 1u : 0u;
    const uint32_t o = warp_reserve(&sh.n_spec, mine);
    uint64_t kmn = ~0ull, kmx = 0ull;
    uint32_t np = 0;
    {
      uint32_t q = o;
#pragma unroll
      for (int j = 0; j < SMALL_EPT; ++j)
        if (x[j] >= theta) {
          const uint64_t k = ckey(km, x[j], (uint32_t)(gbase + tid + NT * j));
          const uint64_t w = weight_A(r, x[j], m);
          ts.K[q] = k;
          ts.W[q] = w;
          ++q;
          kmn = u64min(kmn, k);
          kmx = u64max(kmx, k);
          np += w != 0;
        }
    }
    np = __reduce_add_sync(~0u, np);
    if (lane == 0 && np) atomicAdd(&sh.npass, np);
    __syncthreads();  // keys, weights and the pass count complete
    const int n = (int)sh.n_spec;
    TailScr rs = ts;  // where the rank-ordered keys / weights / prefixes end up
    if (n <= RANK_SMALL) {
      tail_rank_sort(n, ts);
    } else if (small_bucket_sort(r, km, n, ts, sh)) {
      rs.RK = ts.K;
      rs.RW = ts.W;
    } else {  // long runs of ties: buckets of the order key
      tail_gather_end(kmn, kmx, 0u, ts, sh);
      tail_sort(n, ts, sh);
    }
    if (n <= NT) {
      if (tid < 32) tail_resolve_warp(r, sh.u, rs, sh);
      __syncthreads();
    } else {
      tail_resolve(r, sh.u, rs, sh);
    }
    token = sh.res.token;
  }
  if (tid == 0) {
    sh.res.m = m;
    sh.res.greedy = r.greedy;
    sh.res.empty = empty;
    write_row_outputs(p, row, slot, token, status);
  }
  if (debug) {
    __syncthreads();
    const Result res = sh.res;
    const uint32_t kmm = okey(res.m);
#pragma unroll
    for (int j = 0; j < SMALL_EPT; ++j) {
      const int i = tid + NT * j;
      if (i >= V) continue;
      const int64_t o = (int64_t)row * V + i;
      const uint32_t gid = (uint32_t)(gbase + i);
      const float xv = x[j];
      bool kept = false;
      float prob = 0.0f;
      if (!empty && xv == xv) {
        if (one) {
          kept = gid == token;
          prob = kept ? 1.0f : 0.0f;
        } else if (xv > -INFINITY && ckey(kmm, xv, gid) <= res.ckK && weight_A(r, xv, res.m) != 0) {
          kept = true;
          prob = (float)__ddiv_rn((double)spec_w_from_e(spec_e(xv, res.m)), (double)res.WK);
        }
      }
      if (p.out_x) p.out_x[o] = xv;
      if (p.out_kept) p.out_kept[o] = kept ? 1 : 0;
      if (p.out_probs) p.out_probs[o] = prob;
    }
  }
}

// ------------------------------------------------------------ commit

// State updates for ids chosen elsewhere: one thread per row.  Ids outside
// [vocab_offset, vocab_offset + V) change nothing.
__global__ void __launch_bounds__(128) commit_kernel(const mstar_sampler_params_t p, const int64_t *ids) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= p.B) return;
  const int slot = p.slot_idx ? p.slot_idx[row] : row;
  const int64_t id = ids[row];
  if (slot < 0 || id < p.vocab_offset || id >= p.vocab_offset + p.V) return;
  mstar_sampler_params_t q = p;
  q.out_ids = nullptr;
  q.out_ids32 = nullptr;
  q.out_status = nullptr;
  q.uniforms = nullptr;  // (the offset advances when asked to)
  write_row_outputs(q, row, slot, (uint32_t)id, 0u);
}

// ------------------------------------------------------------ TP merge

// One CTA per row: merge tp_world candidate records and sample.
__global__ void __launch_bounds__(NT, 1)
    tp_merge_kernel(const mstar_sampler_params_t p, int tp_cap, int tp_world, int rec_words, int64_t V_global,
                    const uint32_t *recv, uint32_t *pend) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ CtaSh sh;
  const int row = blockIdx.x, tid = threadIdx.x;
  const int slot = p.slot_idx ? p.slot_idx[row] : row;
  if (slot < 0) {
    if (tid == 0) {
      if (p.out_ids) p.out_ids[row] = 0;
      if (p.out_ids32) p.out_ids32[row] = 0;
      if (p.out_status) p.out_status[row] = 0;
      if (pend) pend[2 * row] = 0u;
    }
    return;
  }
  Row r;
  row_init(r, p, row, slot, V_global);
  const TailScr ts = tail_scratch(smem);
  float m = -INFINITY;
  uint32_t status = 0;
  bool partial = false;  // some shard sent only the first tp_cap members of its A set
  for (int q = 0; q < tp_world; ++q) {
    const uint32_t *rec = recv + ((int64_t)q * p.B + row) * rec_words;
    m = fmaxf(m, __uint_as_float(rec[0]));
    status |= rec[2];
    partial |= (rec[3] & 1u) && rec[1] >= (uint32_t)tp_cap;
  }
  status &= ~(uint32_t)MSTAR_STATUS_EMPTY;
  if (partial && !(r.greedy || r.K == 1) && m > -INFINITY) {
    if (pend) {  // decided by the second round: no output and no state update here
      if (tid == 0) {
        pend[2 * row] = 1u;
        pend[2 * row + 1] = __float_as_uint(m);
      }
      return;
    }
    status |= MSTAR_STATUS_TP_OVERFLOW;
  }
  if (pend && tid == 0) pend[2 * row] = 0u;
  if (tid == 0) {
    sh.nloc = 0;
    sh.best = 0xFFFFFFFFu;
    sh.res.token = 0;
    sh.status = 0;
    sh.theta = 0.0f;
    sh.u = p.uniforms ? p.uniforms[row]
                      : philox_uniform(p.seed ? p.seed[slot] : 0ull, p.offset ? p.offset[slot] : 0ull);
    tail_reset(sh);
  }
  const bool empty = !(m > -INFINITY);
  const bool one = r.greedy || r.K == 1;
  if (!empty && tid < 32) {
    const float t = choose_theta(r, m);
    if (tid == 0) sh.theta = t;
  }
  __syncthreads();
  if (!empty) {
    const float theta = sh.theta;
    const uint32_t km = okey(m);
    uint32_t best = 0xFFFFFFFFu;
    uint64_t kmn = ~0ull, kmx = 0ull;
    uint32_t np = 0;
    for (int q = 0; q < tp_world; ++q) {
      const uint32_t *rec = recv + ((int64_t)q * p.B + row) * rec_words;
      const int n = (int)min(rec[1], (uint32_t)tp_cap);
      for (int j = tid; j < n; j += NT) {
        const float x = __uint_as_float(rec[4 + 2 * j]);
        const uint32_t gid = rec[5 + 2 * j];
        if ((int64_t)gid >= V_global) {  // not an id of this vocabulary: the entry is left out
          atomicOr(&sh.status, MSTAR_STATUS_BAD_RECORD);
          continue;
        }
        if (one) {
          if (x == m) best = min(best, gid);
        } else if (x >= theta) {
          const uint32_t idx = atomicAdd(&sh.nloc, 1u);
          if (idx < (uint32_t)TAIL_CAP) tail_put(r, m, km, Cand{x, gid}, (int)idx, ts, kmn, kmx, np);
        }
      }
    }
    if (one) {
      if (best != 0xFFFFFFFFu) atomicMin(&sh.best, best);
      __syncthreads();
      if (tid == 0) sh.res.token = sh.best;
    } else {
      __syncthreads();  // every candidate counted
      tail_finish<0>(r, sh.u, km, (int)min(sh.nloc, (uint32_t)TAIL_CAP), kmn, kmx, np, 0, nullptr, ts, sh);
    }
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t token = sh.res.token;
    status |= sh.status;
    if (empty || (int64_t)token >= V_global) {  // (no valid entry stood)
      status |= MSTAR_STATUS_EMPTY;
      token = 0;
    }
    write_row_outputs(p, row, slot, token, status);
  }
}

// ------------------------------------------------------------ TP, second round
//
// Rows whose shards sent only the first tp_cap members of their A sets
// (top_k off, or above the record capacity) are decided with one more
// exchange.  tp_mass_kernel: each shard's exact A mass against the row max M
// the first merge found (one CTA per deferred row, over the shard values
// its record kernel left in xbuf).  tp_merge2_kernel: with W_A = the sum of
// those masses, the rank-ordered union of the records is exact up to k*,
// the smallest last-sent key among the partial shards (every key up to it
// was sent); the row is decided when its kept set ends there (top_p) or its
// draw point falls there (top_p off), and flagged MSTAR_STATUS_TP_OVERFLOW
// otherwise.  Rows with top_k above the capacity are decided when their
// first K members are all known.

__global__ void __launch_bounds__(NT)
    tp_mass_kernel(const mstar_sampler_params_t p, const float *xbuf, const uint32_t *pend, uint32_t *send2) {
  __shared__ uint64_t part[NWARP];
  const int row = blockIdx.x, tid = threadIdx.x;
  if (!pend[2 * row]) {
    if (tid == 0) {
      send2[2 * row] = 0u;
      send2[2 * row + 1] = 0u;
    }
    return;
  }
  const int slot = p.slot_idx ? p.slot_idx[row] : row;
  Row r;
  row_init(r, p, row, slot, p.V);
  const float M = __uint_as_float(pend[2 * row + 1]);
  const float *x = xbuf + (int64_t)row * p.V;
  uint64_t acc = 0;
  for (int64_t e = tid; e < p.V; e += NT) {
    const float v = x[e];
    if (v == v && v > -INFINITY) acc += weight_A(r, v, M);
  }
  for (int o = 16; o; o >>= 1) acc += (uint64_t)__shfl_xor_sync(~0u, (unsigned long long)acc, o);
  if ((tid & 31) == 0) part[tid >> 5] = acc;
  __syncthreads();
  if (tid == 0) {
    uint64_t t = 0;
    for (int w = 0; w < NWARP; ++w) t += part[w];
    send2[2 * row] = (uint32_t)t;
    send2[2 * row + 1] = (uint32_t)(t >> 32);
  }
}

__global__ void __launch_bounds__(NT, 1)
    tp_merge2_kernel(const mstar_sampler_params_t p, int tp_cap, int tp_world, int rec_words, int64_t V_global,
                     const uint32_t *recv, const uint32_t *recv2, const uint32_t *pend) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ CtaSh sh;
  __shared__ unsigned long long kstar;  // smallest last-sent key among the partial shards
  __shared__ unsigned long long kq[16];
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  if (!pend[2 * row]) return;  // decided by the first merge (or a padding row)
  const int slot = p.slot_idx ? p.slot_idx[row] : row;
  Row r;
  row_init(r, p, row, slot, V_global);
  const TailScr ts = tail_scratch(smem);
  const float m = __uint_as_float(pend[2 * row + 1]);
  const uint32_t km = okey(m);
  uint32_t status = 0;
  for (int q = 0; q < tp_world; ++q) status |= recv[((int64_t)q * p.B + row) * rec_words + 2];
  status &= ~(uint32_t)MSTAR_STATUS_EMPTY;
  if (tid == 0) {
    sh.nloc = 0;
    sh.status = 0;
    sh.theta = 0.0f;
    sh.res.token = 0;
    sh.u = p.uniforms ? p.uniforms[row]
                      : philox_uniform(p.seed ? p.seed[slot] : 0ull, p.offset ? p.offset[slot] : 0ull);
    kstar = ~0ull;
    tail_reset(sh);
  }
  if (tid < 16) kq[tid] = 0ull;
  if (tid < 32) {
    const float t = choose_theta(r, m);
    if (tid == 0) sh.theta = t;
  }
  __syncthreads();
  const float theta = sh.theta;
  uint64_t kmn = ~0ull, kmx = 0ull;
  uint32_t np = 0;
  for (int q = 0; q < tp_world; ++q) {
    const uint32_t *rec = recv + ((int64_t)q * p.B + row) * rec_words;
    const bool part = (rec[3] & 1u) && rec[1] >= (uint32_t)tp_cap;
    const int n = (int)min(rec[1], (uint32_t)tp_cap);
    unsigned long long lastk = 0ull;
    for (int j = tid; j < n; j += NT) {
      const float x = __uint_as_float(rec[4 + 2 * j]);
      const uint32_t gid = rec[5 + 2 * j];
      if ((int64_t)gid >= V_global) {
        atomicOr(&sh.status, MSTAR_STATUS_BAD_RECORD);
        continue;
      }
      if (part) lastk = u64max(lastk, ckey(km, x, gid));
      if (x >= theta) {
        const uint32_t idx = atomicAdd(&sh.nloc, 1u);
        if (idx < (uint32_t)TAIL_CAP) tail_put(r, m, km, Cand{x, gid}, (int)idx, ts, kmn, kmx, np);
      }
    }
    if (part) {
      for (int o = 16; o; o >>= 1) lastk = u64max(lastk, (uint64_t)__shfl_xor_sync(~0u, lastk, o));
      if (lane == 0 && q < 16) atomicMax(&kq[q], lastk);
    }
  }
  __syncthreads();
  if (tid == 0)
    for (int q = 0; q < tp_world && q < 16; ++q) {
      const uint32_t *rec = recv + ((int64_t)q * p.B + row) * rec_words;
      if ((rec[3] & 1u) && rec[1] >= (uint32_t)tp_cap) kstar = u64min(kstar, kq[q]);
    }
  const int n = (int)min(sh.nloc, (uint32_t)TAIL_CAP);
  tail_sort_gathered(r, km, n, kmn, kmx, np, ts, sh);
  if (tid == 0) {
    const int npass = (int)sh.npass;
    // known members of A: a prefix of the rank order (keys up to k*)
    int nk = 0;
    while (nk < npass && ts.RK[nk] <= kstar) ++nk;
    const uint64_t G = nk ? ts.RS[nk - 1] + ts.RW[nk - 1] : 0ull;
    auto S = [&](int j) -> uint64_t { return j < nk ? ts.RS[j] : G; };  // exclusive prefix, j <= nk
    bool ok = nk > 0;
    int nA = nk;
    uint64_t WA = 0;
    if (ok && r.topk) {  // the first K members must all be known
      ok = r.K <= nk;
      nA = r.K;
      if (ok) WA = S(nA);
    } else if (ok) {
      for (int q = 0; q < tp_world; ++q)
        WA += (uint64_t)recv2[2 * ((int64_t)q * p.B + row)] |
              ((uint64_t)recv2[2 * ((int64_t)q * p.B + row) + 1] << 32);
      nA = -1;  // all of A (its end may lie past k*)
    }
    int nK = 0;
    uint64_t WK = 0;
    if (ok && r.topp) {  // kept: j == 0 or S_j < P * W_A; the first j >= 1 with S_j >= thr must be known
      const double thr = __dmul_rn((double)r.P, (double)WA);
      const int lim = nA >= 0 ? nA : nk;
      nK = 0;
      for (int j = 1; j <= lim; ++j)
        if (!((double)S(j) < thr)) {
          nK = j;
          break;
        }
      if (nK == 0 && nA >= 0) nK = nA;  // every one of the first K is kept
      ok = nK > 0;
      if (ok) WK = S(nK);
    } else if (ok) {
      nK = nA >= 0 ? nA : nk;
      WK = nA >= 0 ? S(nA) : WA;
    }
    uint32_t token = (uint32_t)(ts.RK[0] & 0xFFFFFFFFu);
    if (ok && WK > 0) {
      const uint64_t rr = draw_point(sh.u, WK);
      ok = false;
      for (int j = 0; j < nK && j < nk; ++j)
        if (S(j) <= rr && rr < S(j) + ts.RW[j]) {
          token = (uint32_t)(ts.RK[j] & 0xFFFFFFFFu);
          ok = true;
          break;
        }
    } else if (ok) {  // no weight anywhere: the leading member stands
      ok = true;
    }
    status |= sh.status;
    if (!ok) status |= MSTAR_STATUS_TP_OVERFLOW;
    write_row_outputs(p, row, slot, token, status);
  }
}

// ================================================================== host

static thread_local std::string g_last_error;

static int fail(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

static int next_pow2(int v) {
  int c = 1;
  while (c < v) c <<= 1;
  return c;
}

static int validate(const mstar_sampler_params_t *p) {
  if (!p) return fail(MSTAR_ERR_INVALID, "params is NULL");
  if (!p->logits) return fail(MSTAR_ERR_INVALID, "logits is NULL");
  if (p->dtype != MSTAR_DTYPE_F32 && p->dtype != MSTAR_DTYPE_BF16)
    return fail(MSTAR_ERR_INVALID, "dtype must be MSTAR_DTYPE_F32 or MSTAR_DTYPE_BF16");
  if (p->B < 1 || p->B > 65535) return fail(MSTAR_ERR_INVALID, "B must be in [1, 65535]");
  // (general-path histogram mass parts are exact for rows of up to 2^21 ids)
  if (p->V < 1 || p->V > (1 << 21)) return fail(MSTAR_ERR_INVALID, "V must be in [1, 2097152]");
  if (p->ld < p->V) return fail(MSTAR_ERR_INVALID, "ld must be >= V");
  if (p->vocab_offset < 0 || p->vocab_offset + p->V > 0x7FFFFFFFLL)
    return fail(MSTAR_ERR_INVALID, "vocab_offset out of range");
  if (p->num_slots < 1) return fail(MSTAR_ERR_INVALID, "num_slots must be >= 1");
  if (!p->slot_idx && p->num_slots < p->B)
    return fail(MSTAR_ERR_INVALID, "without slot_idx, num_slots must be >= B");
  if (p->hist_ids && p->seen_bits) return fail(MSTAR_ERR_INVALID, "give hist_ids or seen_bits, not both");
  if (p->hist_ids && (!p->hist_len || p->H < 1)) return fail(MSTAR_ERR_INVALID, "hist_ids needs hist_len and H >= 1");
  if (p->seen_bits && p->seen_words * 32 < p->vocab_offset + p->V)
    return fail(MSTAR_ERR_INVALID, "seen_words too small for the vocabulary");
  if (p->allowed_bits && p->allowed_words * 32 < p->vocab_offset + p->V)
    return fail(MSTAR_ERR_INVALID, "allowed_words too small for the vocabulary");
  if ((p->bias_ids == nullptr) != (p->bias_vals == nullptr))
    return fail(MSTAR_ERR_INVALID, "bias_ids and bias_vals go together");
  if (p->bias_ids && p->NB < 1) return fail(MSTAR_ERR_INVALID, "NB must be >= 1 with bias_ids");
  if (!p->uniforms && (!p->seed || !p->offset))
    return fail(MSTAR_ERR_INVALID, "need uniforms, or seed and offset");
  if (!p->out_ids && !p->out_ids32) return fail(MSTAR_ERR_INVALID, "need out_ids or out_ids32");
  if ((p->flags & MSTAR_FLAG_UPDATE_HISTORY) && !p->hist_ids)
    return fail(MSTAR_ERR_INVALID, "UPDATE_HISTORY needs hist_ids");
  if ((p->flags & MSTAR_FLAG_UPDATE_SEEN) && !p->seen_bits)
    return fail(MSTAR_ERR_INVALID, "UPDATE_SEEN needs seen_bits");
  if (p->stop_ids && p->NS < 1) return fail(MSTAR_ERR_INVALID, "NS must be >= 1 with stop_ids");
  if (p->stop_flags && !p->stop_ids) return fail(MSTAR_ERR_INVALID, "stop_flags needs stop_ids");
  return MSTAR_OK;
}

// Device properties the planner reads, cached per device (the calling
// thread's current device; a process may drive several GPUs, possibly of
// different kinds) under one lock.
constexpr int kMaxDevices = 64;
static std::mutex g_dev_mu;

static int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  return dev;
}

static int device_attr(cudaDeviceAttr what, int (&cache)[kMaxDevices], int fallback) {
  const int dev = current_device();
  std::lock_guard<std::mutex> g(g_dev_mu);
  if (cache[dev] <= 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, what, dev) != cudaSuccess || v <= 0) {
      cudaGetLastError();
      v = fallback;
    }
    cache[dev] = v;
  }
  return cache[dev];
}

static int max_smem_optin() {
  static int cache[kMaxDevices] = {};
  return device_attr(cudaDevAttrMaxSharedMemoryPerBlockOptin, cache, 232448);
}

static int sm_count() {
  static int cache[kMaxDevices] = {};
  return device_attr(cudaDevAttrMultiProcessorCount, cache, 148);
}

template <typename T, int MODE>
__global__ void sampler_kernel(const mstar_sampler_params_t p, const Plan pl, uint32_t *tp_send);

// CTAs of the step kernel that can be resident at once with clusters of S
// CTAs and smem bytes of dynamic shared memory each (clusters are placed
// whole, inside one GPC, so the width decides how many SMs a wave can use);
// 0 if the runtime cannot say.  Cached per configuration.
static int resident_ctas(int dtype, int mode, int S, int smem) {
  static int keys[256][5], vals[256], used = 0;
  const int dev = current_device();
  std::lock_guard<std::mutex> g(g_dev_mu);
  for (int i = 0; i < used; ++i)
    if (keys[i][0] == dtype && keys[i][1] == mode && keys[i][2] == S && keys[i][3] == smem && keys[i][4] == dev)
      return vals[i];
  const void *fn = dtype == MSTAR_DTYPE_BF16
                       ? (mode ? (const void *)sampler_kernel<__nv_bfloat16, 1> : (const void *)sampler_kernel<__nv_bfloat16, 0>)
                       : (mode ? (const void *)sampler_kernel<float, 1> : (const void *)sampler_kernel<float, 0>);
  int v = 0;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) == cudaSuccess) v = clusters * S;
  }
  cudaGetLastError();  // a refused query leaves no error behind
  if (used < 256) {
    keys[used][0] = dtype;
    keys[used][1] = mode;
    keys[used][2] = S;
    keys[used][3] = smem;
    keys[used][4] = dev;
    vals[used++] = v;
  }
  return v;
}

static int plan_launch(const mstar_sampler_params_t *p, int mode, int tp_cap, Plan &pl) {
  const int es = p->dtype == MSTAR_DTYPE_BF16 ? 2 : 4;
  // materialized specials: the distinct history ids (at most H) and the bias
  // ids; seen-mask ids are visited from the seen map instead (no bound)
  const int spec_max = (p->hist_ids ? p->H : 0) + (p->bias_ids ? p->NB : 0);
  const int spec_cap = std::max(16, spec_max);
  const int ht_cap = next_pow2(std::max(32, 2 * spec_cap));
  const int static_bytes = (int)sizeof(CtaSh);
  const int budget = max_smem_optin() - static_bytes - 1024;
  auto need = [&](int s, Plan &q) {
    int64_t slice = (p->V + s - 1) / s;
    slice = (slice + 63) / 64 * 64;
    q.S = s;
    q.es = es;
    q.slice = slice;
    const int64_t span_bytes = slice * es + 32;
    q.data_bytes = (int)std::max<int64_t>(LEAN_SCRATCH, (span_bytes + 127) / 128 * 128);
    const int64_t nvec = (span_bytes + 15) / 16;
    const int64_t positions = nvec * (16 / es);
    q.map_bytes = (int)(((positions + 31) / 32) * 4);
    q.map_bytes = (q.map_bytes + 127) / 128 * 128;
    q.seen_map = p->seen_bits ? 1 : 0;
    q.ht_cap = ht_cap;
    q.spec_cap = spec_cap;
    const int work = q.map_bytes * (1 + q.seen_map) + std::max(WORK_BYTES_MIN, ht_cap * 8 + NBIN * 4);
    q.off_work = q.data_bytes;
    q.off_spec = q.off_work + (work + 127) / 128 * 128;
    q.off_lcand = q.off_spec + (spec_cap * 8 + 127) / 128 * 128;
    q.off_bias = q.off_lcand + TAIL_CAP * 8;
    const int bias_bytes = p->bias_ids && p->NB <= BIAS_SMEM ? BIAS_SMEM * 8 : 0;
    q.smem_bytes = q.off_bias + bias_bytes;
    q.mode = mode;
    q.tp_cap = tp_cap;
    q.rec_words = 4 + 2 * tp_cap;
    return q.smem_bytes <= budget && slice * es <= (int64_t)MAX_CHUNKS * CHUNK_BYTES;
  };
  if (p->cluster_size > 0) {
    if (p->cluster_size > 16) return fail(MSTAR_ERR_INVALID, "cluster_size must be <= 16");
    if (!need(p->cluster_size, pl)) return fail(MSTAR_ERR_UNSUPPORTED, "row does not fit the requested cluster size");
    return MSTAR_OK;
  }
  // the smallest cluster the row fits with slices of at most NVR vectors
  // per thread (else the smallest it fits at all), widened while the grid leaves
  // SMs idle (small batches: each row's slice is then streamed by more SMs),
  // up to the portable cluster size and keeping slices >= 8192 elements
  auto in_tile = [&](int s) {
    const int64_t slice = ((p->V + s - 1) / s + 63) / 64 * 64;
    return slice * es <= (int64_t)NT * NVR * 16;
  };
  int smin = 0;
  for (int s = 1; s <= 16 && !smin; ++s)
    if (in_tile(s) && need(s, pl)) smin = s;
  for (int s = 1; s <= 16 && !smin; ++s)
    if (need(s, pl)) smin = s;
  if (!smin) return fail(MSTAR_ERR_UNSUPPORTED, "row too large for a 16-CTA cluster");
  if ((int64_t)p->B * smin > (int64_t)sm_count() && smin < 8) {
    // more than one wave: the portable width that keeps the most CTAs
    // resident (ties: the narrower); e.g. clusters of 7 leave a fifth of
    // the SMs idle where clusters of 8 do not
    int best = smin, best_ctas = resident_ctas(p->dtype, mode, smin, pl.smem_bytes);
    for (int s = smin + 1; s <= 8 && best_ctas > 0; ++s) {
      Plan q;
      if (!need(s, q)) continue;
      const int c = resident_ctas(p->dtype, mode, s, q.smem_bytes);
      if (c > best_ctas) {
        best = s;
        best_ctas = c;
      }
    }
    need(best, pl);
    return MSTAR_OK;
  }
  int target = std::min(8, std::max(1, sm_count() / std::max(1, p->B)));
  target = (int)std::min<int64_t>(target, std::max<int64_t>(1, p->V / 8192));
  for (int s = std::max(smin, target); s > smin; --s)
    if (need(s, pl)) return MSTAR_OK;
  need(smin, pl);
  return MSTAR_OK;
}

template <typename T, int MODE>
static int launch_T(const mstar_sampler_params_t *p, const Plan &pl, uint32_t *send, cudaStream_t st) {
  auto kern = sampler_kernel<T, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem_bytes);
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  if (pl.S > 8) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess)
      return fail(MSTAR_ERR_CUDA, std::string("non-portable cluster: ") + cudaGetErrorString(e));
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.S, p->B, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = pl.smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = pl.S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // blocks may be placed while the previous kernel of the stream finishes;
  // the kernel waits for it (griddepcontrol.wait) before reading its inputs
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, *p, pl, send);
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return MSTAR_OK;
}

// Small rows (V <= SMALL_V, automatic width, no testing flags): the
// one-CTA-per-row kernel.
static bool use_small(const mstar_sampler_params_t *p, int mode) {
  return mode == 0 && p->V <= SMALL_V && p->cluster_size == 0 &&
         !(p->flags & (MSTAR_FLAG_FORCE_GENERAL | MSTAR_FLAG_TEST_WITHHOLD));
}

template <typename T>
static int launch_small(const mstar_sampler_params_t *p, cudaStream_t st) {
  auto kern = small_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMALL_SMEM);
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p->B, 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = SMALL_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, *p);
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return MSTAR_OK;
}

static int launch(const mstar_sampler_params_t *p, int mode, int tp_cap, uint32_t *send, cudaStream_t st,
                  float *xdump = nullptr) {
  if (use_small(p, mode))
    return p->dtype == MSTAR_DTYPE_BF16 ? launch_small<__nv_bfloat16>(p, st) : launch_small<float>(p, st);
  Plan pl{};
  int rc = plan_launch(p, mode, tp_cap, pl);
  if (rc) return rc;
  pl.xdump = xdump;
  if (p->dtype == MSTAR_DTYPE_BF16)
    return mode == 0 ? launch_T<__nv_bfloat16, 0>(p, pl, send, st) : launch_T<__nv_bfloat16, 1>(p, pl, send, st);
  return mode == 0 ? launch_T<float, 0>(p, pl, send, st) : launch_T<float, 1>(p, pl, send, st);
}

#include "lmhead.cuh"

}  // namespace mstar

using namespace mstar;

extern "C" {

int mstar_sampler_abi_version(void) { return MSTAR_SAMPLER_ABI_VERSION; }

const char *mstar_sampler_last_error(void) { return g_last_error.c_str(); }

int mstar_sampler_plan(const mstar_sampler_params_t *p, int32_t *cluster_size, int64_t *smem_bytes) {
  int rc = validate(p);
  if (rc) return rc;
  if (use_small(p, 0)) {
    if (cluster_size) *cluster_size = 1;
    if (smem_bytes) *smem_bytes = SMALL_SMEM;
    return MSTAR_OK;
  }
  Plan pl{};
  rc = plan_launch(p, 0, 0, pl);
  if (rc) return rc;
  if (cluster_size) *cluster_size = pl.S;
  if (smem_bytes) *smem_bytes = pl.smem_bytes;
  return MSTAR_OK;
}

int mstar_sampler_step(const mstar_sampler_params_t *p, void *stream) {
  int rc = validate(p);
  if (rc) return rc;
  return launch(p, 0, 0, nullptr, static_cast<cudaStream_t>(stream));
}

int32_t mstar_sampler_tp_record_words(int32_t tp_cap) { return 4 + 2 * tp_cap; }

static int tp_local_impl(const mstar_sampler_params_t *p, int32_t tp_cap, uint32_t *send, float *xbuf,
                         void *stream) {
  if (!p) return fail(MSTAR_ERR_INVALID, "params is NULL");
  mstar_sampler_params_t q = *p;
  if (!q.out_ids && !q.out_ids32) q.out_ids32 = reinterpret_cast<int32_t *>(send);  // not written in TP mode
  int rc = validate(&q);
  if (rc) return rc;
  if (!send) return fail(MSTAR_ERR_INVALID, "send is NULL");
  if (tp_cap < 1 || tp_cap > TAIL_CAP) return fail(MSTAR_ERR_INVALID, "tp_cap must be in [1, 2048]");
  if (q.out_x || q.out_kept || q.out_probs)
    return fail(MSTAR_ERR_UNSUPPORTED, "dense debug outputs are single-shard only");
  q.flags &= ~(MSTAR_FLAG_UPDATE_HISTORY | MSTAR_FLAG_UPDATE_SEEN | MSTAR_FLAG_ADVANCE_OFFSET);
  return launch(&q, 1, tp_cap, send, static_cast<cudaStream_t>(stream), xbuf);
}

int mstar_sampler_tp_local(const mstar_sampler_params_t *p, int32_t tp_cap, uint32_t *send, void *stream) {
  return tp_local_impl(p, tp_cap, send, nullptr, stream);
}

int mstar_sampler_tp_local2(const mstar_sampler_params_t *p, int32_t tp_cap, uint32_t *send, float *xbuf,
                            void *stream) {
  if (!xbuf) return fail(MSTAR_ERR_INVALID, "xbuf is NULL");
  return tp_local_impl(p, tp_cap, send, xbuf, stream);
}

int64_t mstar_lmhead_workspace_bytes(int32_t B) {
  if (B < 1 || B > lmh::MAX_N) return -1;
  return lmh::workspace_bytes(B);
}

int mstar_lmhead_logits(const void *hidden, const void *weight, int32_t B, int32_t V, int32_t d, void *logits,
                        int32_t dtype, int64_t ld, void *workspace, int64_t workspace_bytes, uint32_t *status,
                        void *stream) {
  return lmh::logits(hidden, weight, B, V, d, logits, dtype, ld, workspace, workspace_bytes, status,
                     static_cast<cudaStream_t>(stream));
}

int mstar_lmhead_logits_static(const void *hidden, const void *weight, int32_t B, int32_t V, int32_t d,
                               void *logits, int32_t dtype, int64_t ld, uint32_t *status, void *stream) {
  return lmh::logits_static(hidden, weight, B, V, d, logits, dtype, ld, status, static_cast<cudaStream_t>(stream));
}

int mstar_sampler_lmhead_step(const mstar_sampler_params_t *p, const void *hidden, const void *weight, int32_t d,
                              void *workspace, int64_t workspace_bytes, uint32_t *status, void *stream) {
  int rc = validate(p);
  if (rc) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = lmh::logits(hidden, weight, p->B, p->V, d, const_cast<void *>(p->logits), p->dtype, p->ld, workspace,
                   workspace_bytes, status, st);
  if (rc) return rc;
  return launch(p, 0, 0, nullptr, st);
}

int mstar_sampler_commit(const mstar_sampler_params_t *p, const int64_t *ids, void *stream) {
  if (!p) return fail(MSTAR_ERR_INVALID, "params is NULL");
  if (!ids) return fail(MSTAR_ERR_INVALID, "ids is NULL");
  if (p->B < 1 || p->B > (1 << 24)) return fail(MSTAR_ERR_INVALID, "B must be in [1, 2^24]");
  if (p->V < 1 || p->vocab_offset < 0 || p->vocab_offset + p->V > 0x7FFFFFFFLL)
    return fail(MSTAR_ERR_INVALID, "V / vocab_offset out of range");
  if (p->num_slots < 1 || (!p->slot_idx && p->num_slots < p->B))
    return fail(MSTAR_ERR_INVALID, "num_slots must cover the rows");
  if ((p->flags & MSTAR_FLAG_UPDATE_HISTORY) && (!p->hist_ids || !p->hist_len || p->H < 1))
    return fail(MSTAR_ERR_INVALID, "UPDATE_HISTORY needs hist_ids, hist_len and H >= 1");
  if ((p->flags & MSTAR_FLAG_UPDATE_SEEN) && (!p->seen_bits || p->seen_words * 32 < p->vocab_offset + p->V))
    return fail(MSTAR_ERR_INVALID, "UPDATE_SEEN needs seen_bits covering the vocabulary");
  if ((p->flags & MSTAR_FLAG_ADVANCE_OFFSET) && !p->offset)
    return fail(MSTAR_ERR_INVALID, "ADVANCE_OFFSET needs offset");
  if (p->stop_ids && p->NS < 1) return fail(MSTAR_ERR_INVALID, "NS must be >= 1 with stop_ids");
  if (p->stop_flags && !p->stop_ids) return fail(MSTAR_ERR_INVALID, "stop_flags needs stop_ids");
  commit_kernel<<<(p->B + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(*p, ids);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return MSTAR_OK;
}

static int tp_merge_check(const mstar_sampler_params_t *p, int32_t tp_cap, int32_t tp_world, int64_t V_global,
                          const void *recv) {
  int rc = validate(p);
  if (rc) return rc;
  if (!recv) return fail(MSTAR_ERR_INVALID, "recv is NULL");
  if (tp_world < 1 || tp_world * tp_cap > TAIL_CAP)
    return fail(MSTAR_ERR_INVALID, "tp_world * tp_cap must be in [1, 2048]");
  if (V_global < p->V || V_global > (1 << 21) * (int64_t)tp_world)
    return fail(MSTAR_ERR_INVALID, "V_global must be in [V, tp_world * 2^21]");
  // the merged id may come from any rank's shard: per-slot state indexed by
  // the global id must cover the whole vocabulary
  if (p->seen_bits && p->seen_words * 32 < V_global)
    return fail(MSTAR_ERR_INVALID, "seen_words too small for V_global");
  return MSTAR_OK;
}

static int tp_merge_impl(const mstar_sampler_params_t *p, int32_t tp_cap, int32_t tp_world, int64_t V_global,
                         const uint32_t *recv, uint32_t *pend, void *stream) {
  int rc = tp_merge_check(p, tp_cap, tp_world, V_global, recv);
  if (rc) return rc;
  const int smem = LEAN_SCRATCH;
  cudaError_t e = cudaFuncSetAttribute(tp_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  tp_merge_kernel<<<p->B, NT, smem, static_cast<cudaStream_t>(stream)>>>(*p, tp_cap, tp_world, 4 + 2 * tp_cap,
                                                                         V_global, recv, pend);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return MSTAR_OK;
}

int mstar_sampler_tp_merge(const mstar_sampler_params_t *p, int32_t tp_cap, int32_t tp_world, int64_t V_global,
                           const uint32_t *recv, void *stream) {
  return tp_merge_impl(p, tp_cap, tp_world, V_global, recv, nullptr, stream);
}

int mstar_sampler_tp_merge1(const mstar_sampler_params_t *p, int32_t tp_cap, int32_t tp_world, int64_t V_global,
                            const uint32_t *recv, uint32_t *pend, void *stream) {
  if (!pend) return fail(MSTAR_ERR_INVALID, "pend is NULL");
  if (tp_world > 16) return fail(MSTAR_ERR_INVALID, "the two-round exchange takes at most 16 ranks");
  return tp_merge_impl(p, tp_cap, tp_world, V_global, recv, pend, stream);
}

int mstar_sampler_tp_mass(const mstar_sampler_params_t *p, const float *xbuf, const uint32_t *pend, uint32_t *send2,
                          void *stream) {
  if (!p) return fail(MSTAR_ERR_INVALID, "params is NULL");
  if (!xbuf || !pend || !send2) return fail(MSTAR_ERR_INVALID, "xbuf, pend and send2 must not be NULL");
  mstar_sampler_params_t q = *p;
  if (!q.out_ids && !q.out_ids32) q.out_ids32 = reinterpret_cast<int32_t *>(send2);  // (no id is written)
  const int rc = validate(&q);
  if (rc) return rc;
  tp_mass_kernel<<<p->B, NT, 0, static_cast<cudaStream_t>(stream)>>>(q, xbuf, pend, send2);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return MSTAR_OK;
}

int mstar_sampler_tp_merge2(const mstar_sampler_params_t *p, int32_t tp_cap, int32_t tp_world, int64_t V_global,
                            const uint32_t *recv, const uint32_t *recv2, const uint32_t *pend, void *stream) {
  int rc = tp_merge_check(p, tp_cap, tp_world, V_global, recv);
  if (rc) return rc;
  if (!recv2 || !pend) return fail(MSTAR_ERR_INVALID, "recv2 and pend must not be NULL");
  if (tp_world > 16) return fail(MSTAR_ERR_INVALID, "the two-round exchange takes at most 16 ranks");
  const int smem = LEAN_SCRATCH;
  cudaError_t e = cudaFuncSetAttribute(tp_merge2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  tp_merge2_kernel<<<p->B, NT, smem, static_cast<cudaStream_t>(stream)>>>(*p, tp_cap, tp_world, 4 + 2 * tp_cap,
                                                                          V_global, recv, recv2, pend);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return MSTAR_OK;
}

float mstar_sampler_philox_uniform(uint64_t seed, uint64_t offset) {
  uint32_t c0 = (uint32_t)offset, c1 = (uint32_t)(offset >> 32), c2 = 0u, c3 = 0u;
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  for (int i = 0; i < 10; ++i) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0, n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    c1 = (uint32_t)p1;
    c3 = (uint32_t)p0;
    c0 = n0;
    c2 = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return (float)(c0 >> 8) * 0x1.0p-24f;
}

}  // extern "C"
