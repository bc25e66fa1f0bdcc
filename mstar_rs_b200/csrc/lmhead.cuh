// LM-head projection on the 5th-generation tensor cores, feeding the sampler.
//
// logits[b, v] = sum_k hidden[b, k] * weight[v, k]: hidden [B, d] and weight
// [V, d] bf16 row-major (the lm_head Linear's layout), fp32 accumulation.
// The call sites this serves project the last hidden state and sample at
// once (python/mstar_rs/models/orpheus.py:349-350,
// python/mstar_rs/models/qwen3_omni.py:517-518).
//
// With B <= 256 the product is a skinny GEMM whose cost is the weight stream
// (V * d * 2 bytes, each byte read once), so the kernel is built around
// keeping that stream at HBM rate on every SM until the end.  One persistent
// CTA per SM takes an equal, contiguous share of the (vocabulary tile of BM
// ids, k-block of BK) units (stream-K): 151936 ids make 1187 tiles, which
// whole-tile shares would spread as 9 or 8 per SM.  A tile split between
// CTAs is finished by the CTA holding its first k-blocks, which adds the
// fp32 partial sums the later CTAs left in the workspace (one slot and one
// ready flag per CTA; a CTA's only partial tile is its first segment, which
// it finishes first, so the owner, which reaches the tile last, rarely
// waits).  Without a workspace the shares are whole tiles.  Roles:
//   warp 0    TMA producer: 2-D tensor copies of the weight tile [BM x BK]
//             and the hidden tile [N x BK] of each k-block, as 64-wide
//             boxes, into a ring of stages (128-byte swizzled rows, the
//             layout the MMA descriptors name); the first ring is issued
//             before the CTA's set-up barrier;
//   warp 1    MMA issuer: tcgen05.mma kind::f16 (M = BM vocabulary ids,
//             N = batch rows padded to 16, K = 16 per instruction) into one
//             of two TMEM accumulators, so the epilogue of tile t overlaps
//             the MMAs of tile t + grid; owns the TMEM allocation;
//   warps 2-5 epilogue: tcgen05.ld of the accumulator (TMEM lane = vocab id,
//             column = batch row) and the per-tile work.
// Every wait is bounded (mbar_wait); a wait that runs out raises an error
// word, every role stops issuing, drains what it issued and the CTA exits.

namespace lmh {

constexpr int BM = 128;          // vocabulary ids per tile (MMA M, TMEM lanes)
constexpr int BOX_K = 64;        // hidden elements per TMA box: one 128-byte swizzle row
// A k-block (one pipeline stage) is two adjacent boxes: 256 contiguous bytes
// of every weight row, one L2 256-byte promotion, so each DRAM access the
// stream makes serves a whole stage instead of half of it (one box per
// stage streamed at 5.5 TB/s, two at 6.1 TB/s; B=64, V=151936, d=2048).
constexpr int KBOXES = 2;
constexpr int BK = BOX_K * KBOXES;  // hidden elements per k-block
constexpr int THREADS = 192;     // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int MAX_STAGES = 12;
constexpr int MAX_N = 256;       // batch rows per launch (MMA N limit)
constexpr int A_BYTES = BM * BK * 2;  // 32 KB of weight rows per stage
constexpr int A_BOX = BM * BOX_K * 2;  // one weight box (16 KB)
constexpr int SMEM_BUDGET = 220 * 1024;

// Error word bits (the epilogue reports them per launch).
constexpr uint32_t ERR_TIMEOUT = 1u;

struct Gemm {
  int B, V, d, N;       // N: B rounded up to a multiple of 16
  int nkb, ntiles, stages;
  void *out;            // logits [B, ld] (dtype), or NULL
  int64_t ld;
  int out_dtype;        // MSTAR_DTYPE_F32 / MSTAR_DTYPE_BF16
  uint32_t *err;        // error word in global memory, or NULL
  float *ws;            // partial-tile slots [grid][N][BM] fp32, or NULL (whole-tile shares)
  uint32_t *flags;      // [grid] ready flags (zero at launch)
};

// First (tile, k-block) unit of CTA c's share; unit u is k-block u % nkb of
// tile u / nkb.  Shares are equal to within one unit (whole tiles without
// a workspace).
__device__ __forceinline__ uint32_t unit_start(const Gemm &g, int c) {
  if (g.ws) return (uint32_t)((uint64_t)g.ntiles * (uint64_t)g.nkb * (uint64_t)c / gridDim.x);
  return (uint32_t)((uint64_t)g.ntiles * (uint64_t)c / gridDim.x) * (uint32_t)g.nkb;
}

// Walks this CTA's share as segments: k-blocks [k0, k1) of one tile.
struct Work {
  uint32_t u, u1;
  int tile, k0, k1;
  __device__ explicit Work(const Gemm &g) : u(unit_start(g, blockIdx.x)), u1(unit_start(g, blockIdx.x + 1)) {}
  __device__ bool next(const Gemm &g) {
    if (u >= u1) return false;
    tile = (int)(u / (uint32_t)g.nkb);
    k0 = (int)(u % (uint32_t)g.nkb);
    k1 = min(g.nkb, k0 + (int)(u1 - u));
    u += (uint32_t)(k1 - k0);
    return true;
  }
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// L2 eviction policies: the weight stream is read once per step (first out);
// the hidden tile is re-read by every CTA and the logits are read back by
// the sampler right after (last out), so a step's logits stay in the 126 MB
// L2 instead of making a round trip through HBM.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tensor copy global -> shared of box (x, y) of `map` under L2 policy
// `pol`, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                            uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void st_last(float *p, float v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(p), "f"(v), "l"(pol) : "memory");
}
__device__ __forceinline__ void st_last(__nv_bfloat16 *p, __nv_bfloat16 v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.b16 [%0], %1, %2;" ::"l"(p), "h"(__bfloat16_as_ushort(v)), "l"(pol)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile stored as
// 128-byte rows with the 128-byte swizzle, 8-row groups 1024 bytes apart
// (what a TMA box of 64 bf16 x rows with CU_TENSOR_MAP_SWIZZLE_128B
// writes).  Fields: start address >> 4 (bits 0-13), leading byte offset
// (16-29; unused for swizzled K-major, 1), stride byte offset >> 4 (32-45),
// descriptor version 1 (46-47), layout SWIZZLE_128B = 2 (61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and
// B bf16 (7-9 = 1, 10-12 = 1), both K-major (15, 16 = 0), N >> 3 (17-22),
// M >> 4 (24-28).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued is done.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 16 consecutive fp32 columns of this warp's 32 TMEM lanes (one per thread).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__host__ __device__ constexpr int tmem_cols(int N) {  // two accumulators, a power of two >= 32
  int c = 32;
  while (c < 2 * N) c <<= 1;
  return c;
}

// Ready flags of the partial-tile slots (global memory, device scope).
__device__ __forceinline__ void flag_release(uint32_t *f) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(f), "r"(1u) : "memory");
}
__device__ __forceinline__ uint32_t flag_acquire(const uint32_t *f) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
// Bounded wait (kWaitNs) for a flag to be raised; false if the limit ran out.
__device__ __forceinline__ bool flag_wait(const uint32_t *f) {
  uint64_t t0 = 0;
  for (unsigned i = 0; i < kWaitIters; ++i) {
    if (flag_acquire(f)) return true;
    const uint64_t t = global_ns();
    if (i == 0) t0 = t;
    else if (t - t0 > kWaitNs) return false;
    __nanosleep(64);
  }
  return false;
}
// Barrier over the four epilogue warps (named barrier 1), and-reducing `v`.
__device__ __forceinline__ int epilogue_all(int v) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.s32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(v)
      : "memory");
  return r;
}

// Shared state of one CTA.
struct Sh {
  uint64_t full[MAX_STAGES], empty[MAX_STAGES];
  uint64_t tfull[2], tempty[2], mma_done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool aborted(const Sh &sh) { return *reinterpret_cast<const volatile int *>(&sh.abort); }

__device__ __forceinline__ void raise(const Gemm &g, Sh &sh, uint32_t bits) {
  *reinterpret_cast<volatile int *>(&sh.abort) = 1;
  if (g.err) atomicOr(g.err, bits);
}

// Producer: one thread.  k-block `it` (counted across this CTA's share) uses
// stage it % stages; its fill waits for the MMA commit that released the
// stage's previous use.  Resumable: the first `stages` k-blocks are issued
// before the CTA's set-up barrier (no stage has been used yet, so no wait),
// the rest after it.
struct Producer {
  Work w;
  int tile = 0, kb = 0, k1 = 0;
  uint32_t it = 0, armed = 0, armed_par = 0;
  __device__ explicit Producer(const Gemm &g) : w(g) {}
  __device__ bool next(const Gemm &g) {  // the next k-block to load, if any
    if (kb >= k1) {
      if (!w.next(g)) return false;
      tile = w.tile;
      kb = w.k0;
      k1 = w.k1;
    }
    return true;
  }
};

__device__ void produce(const Gemm &g, Sh &sh, uint8_t *sA, uint8_t *sB, const CUtensorMap *tw,
                        const CUtensorMap *th, Producer &P, uint32_t limit) {
  const uint32_t bbytes = (uint32_t)g.N * BK * 2;
  const uint64_t pw = policy_evict_first(), ph = policy_evict_last();
  while (P.it < limit && !aborted(sh) && P.next(g)) {
    const uint32_t s = P.it % (uint32_t)g.stages, use = P.it / (uint32_t)g.stages;
    if (use > 0 && !mbar_wait(&sh.empty[s], (use - 1) & 1u)) {
      raise(g, sh, ERR_TIMEOUT);
      break;
    }
    mbar_expect_tx(&sh.full[s], (uint32_t)A_BYTES + bbytes);
#pragma unroll
    for (int j = 0; j < KBOXES; ++j) {
      tma_load_2d(sA + (size_t)s * A_BYTES + j * A_BOX, tw, P.kb * BK + j * BOX_K, P.tile * BM, &sh.full[s], pw);
      tma_load_2d(sB + (size_t)s * bbytes + j * (bbytes / KBOXES), th, P.kb * BK + j * BOX_K, 0, &sh.full[s], ph);
    }
    P.armed |= 1u << s;
    P.armed_par = (P.armed_par & ~(1u << s)) | ((use & 1u) << s);
    ++P.kb;
    ++P.it;
  }
}

// Every copy issued lands before the CTA may exit (normally long done).
__device__ void produce_drain(const Gemm &g, Sh &sh, const Producer &P) {
  for (int s = 0; s < g.stages; ++s)
    if ((P.armed >> s) & 1u)
      if (!mbar_wait(&sh.full[s], (P.armed_par >> s) & 1u)) raise(g, sh, ERR_TIMEOUT);
}

// MMA issuer: one thread.  Segment number sl of this CTA accumulates into
// TMEM columns (sl & 1) * N; the epilogue frees them (tempty) before reuse.
__device__ void mma_issue(const Gemm &g, Sh &sh, uint8_t *sA, uint8_t *sB, uint32_t tbase) {
  const uint32_t bbytes = (uint32_t)g.N * BK * 2;
  const uint32_t idesc = idesc_bf16(BM, g.N);
  const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
  uint32_t it = 0, tl = 0;
  Work w(g);
  for (; !aborted(sh) && w.next(g); ++tl) {
    const uint32_t acc = tl & 1u, use = tl >> 1;
    if (use > 0 && !mbar_wait(&sh.tempty[acc], (use - 1) & 1u)) {
      raise(g, sh, ERR_TIMEOUT);
      break;
    }
    tc_fence_after();
    const uint32_t dcol = tbase + acc * (uint32_t)g.N;
    bool ok = true;
    for (int kb = w.k0; kb < w.k1; ++kb, ++it) {
      const uint32_t s = it % (uint32_t)g.stages;
      if (!mbar_wait(&sh.full[s], (it / (uint32_t)g.stages) & 1u)) {
        raise(g, sh, ERR_TIMEOUT);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t as = a0 + s * (uint32_t)A_BYTES, bs = b0 + s * bbytes;
#pragma unroll
      for (int j = 0; j < KBOXES; ++j)
#pragma unroll
        for (int k = 0; k < BOX_K / 16; ++k)  // K = 16 bf16 = 32 bytes per instruction
          mma_bf16(dcol, sw128_desc(as + j * A_BOX + 32u * k), sw128_desc(bs + j * (bbytes / KBOXES) + 32u * k),
                   idesc, (kb != w.k0 || j || k) ? 1u : 0u);
      mma_commit(&sh.empty[s]);
    }
    if (!ok) break;
    mma_commit(&sh.tfull[acc]);
  }
  // every MMA issued is complete before TMEM is released
  mma_commit(&sh.mma_done);
  if (!mbar_wait(&sh.mma_done, 0)) raise(g, sh, ERR_TIMEOUT);
}

}  // namespace lmh

// Plain projection: the epilogue writes logits (fp32 or bf16, rounded to
// nearest even) to out[b * ld + v].
__global__ void __launch_bounds__(lmh::THREADS, 1)
    lmhead_gemm_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap th,
                       const lmh::Gemm g) {
  using namespace lmh;
  extern __shared__ __align__(1024) uint8_t lm_smem_raw[];
  __shared__ Sh sh;
  uint8_t *smem = lm_smem_raw + ((1024u - (smem_u32(lm_smem_raw) & 1023u)) & 1023u);
  uint8_t *sA = smem, *sB = smem + (size_t)g.stages * A_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncols = tmem_cols(g.N);
  // a dependent launch (the sampler step) may be scheduled as CTAs finish;
  // its griddepcontrol.wait still waits for this whole grid and its writes
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  Producer P(g);
  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&th)) : "memory");
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh.tfull[a], 1);
      mbar_init(&sh.tempty[a], 4);  // one arrive per epilogue warp
    }
    mbar_init(&sh.mma_done, 1);
    sh.abort = 0;
    fence_barrier_init();
    produce(g, sh, sA, sB, &tw, &th, P, (uint32_t)g.stages);  // the first ring, while TMEM is allocated
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem_base)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sh.tmem_base;
  if (warp == 0) {
    if (lane == 0) {
      produce(g, sh, sA, sB, &tw, &th, P, 0xFFFFFFFFu);
      produce_drain(g, sh, P);
    }
  } else if (warp == 1) {
    if (lane == 0) mma_issue(g, sh, sA, sB, tbase);
  } else {
    const int quad = warp & 3;  // TMEM lanes 32 * quad .. + 31 belong to this warp
    const int row = quad * 32 + lane;
    const int et = threadIdx.x - 64;  // 0 .. 127 over the epilogue warps
    const uint64_t pol = policy_evict_last();
    uint32_t tl = 0;
    Work w(g);
    for (; w.next(g); ++tl) {
      const uint32_t acc = tl & 1u;
      // one thread waits and the four warps take its verdict together: every
      // later epilogue barrier is then reached by all of them or none, and
      // the tcgen05.ld below is warp-collective
      int go = 1;
      if (et == 0) {
        go = !aborted(sh);
        if (go && !mbar_wait(&sh.tfull[acc], (tl >> 1) & 1u)) {
          raise(g, sh, ERR_TIMEOUT);
          go = 0;
        }
      }
      if (!epilogue_all(go)) break;
      const bool part = w.k0 > 0;               // a later part: leave the partial sums
      const bool owner_split = !part && w.k1 < g.nkb;  // the first part: add the later ones
      // the later parts of this tile are the first segments of the CTAs whose
      // shares start inside it
      const uint32_t tile_end = (uint32_t)(w.tile + 1) * (uint32_t)g.nkb;
      int c_hi = blockIdx.x + 1;
      if (owner_split)
        while (c_hi < (int)gridDim.x && unit_start(g, c_hi) < tile_end) ++c_hi;
      if (owner_split) {
        int ok = 1;
        if (et == 0)
          for (int c = blockIdx.x + 1; c < c_hi && ok; ++c) ok = flag_wait(&g.flags[c]);
        ok = epilogue_all(ok);
        if (!ok) {
          if (et == 0) raise(g, sh, ERR_TIMEOUT);
          break;
        }
        for (int c = blockIdx.x + 1; c < c_hi; ++c) flag_acquire(&g.flags[c]);
      }
      tc_fence_after();
      const int v = w.tile * BM + row;
      const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + acc * (uint32_t)g.N;
      float *slot = part ? g.ws + (size_t)blockIdx.x * (size_t)g.N * BM : nullptr;
      for (int c0 = 0; c0 < g.N; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + (uint32_t)c0, r);
        tmem_wait_ld();
        if (part) {
#pragma unroll
          for (int j = 0; j < 16; ++j) slot[(size_t)(c0 + j) * BM + row] = __uint_as_float(r[j]);
          continue;
        }
        float x[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = __uint_as_float(r[j]);
        for (int c = blockIdx.x + 1; c < c_hi; ++c) {  // partial sums in CTA order
          const float *ps = g.ws + (size_t)c * (size_t)g.N * BM;
#pragma unroll
          for (int j = 0; j < 16; ++j) x[j] += ps[(size_t)(c0 + j) * BM + row];
        }
        if (v < g.V && g.out) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int b = c0 + j;
            if (b >= g.B) break;
            if (g.out_dtype == MSTAR_DTYPE_BF16)
              st_last(static_cast<__nv_bfloat16 *>(g.out) + (int64_t)b * g.ld + v, __float2bfloat16_rn(x[j]), pol);
            else
              st_last(static_cast<float *>(g.out) + (int64_t)b * g.ld + v, x[j], pol);
          }
        }
      }
      if (part) {  // publish the partial sums
        __threadfence();
        epilogue_all(1);
        if (et == 0) flag_release(&g.flags[blockIdx.x]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(ncols) : "memory");
  }
}

// ------------------------------------------------------------ host side

namespace lmh {

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, fetched through the runtime once (the
// library links no driver stub).
static EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
    else
      cudaGetLastError();
  });
  return fn;
}

// Tensor map of a K-major bf16 matrix [rows, d] (row stride d) read as
// boxes of BOX_K x box_rows with the 128-byte swizzle; rows and columns past
// the end read as zeros.
static int make_map(CUtensorMap *m, const void *ptr, int64_t rows, int d, int box_rows) {
  const EncodeTiled enc = encode_fn();
  if (!enc) return fail(MSTAR_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)d * 2u};
  const cuuint32_t box[2] = {(cuuint32_t)BOX_K, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1u, 1u};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MSTAR_ERR_CUDA, "cuTensorMapEncodeTiled failed, code " + std::to_string((int)r));
  return MSTAR_OK;
}

static int check_operands(const void *hidden, const void *weight, int B, int V, int d) {
  if (!hidden || !weight) return fail(MSTAR_ERR_INVALID, "hidden and weight must not be NULL");
  if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(weight)) & 15u)
    return fail(MSTAR_ERR_INVALID, "hidden and weight must be 16-byte aligned");
  if (B < 1 || B > MAX_N) return fail(MSTAR_ERR_INVALID, "B must be in [1, 256]");
  if (V < 1 || V > (1 << 21)) return fail(MSTAR_ERR_INVALID, "V must be in [1, 2097152]");
  if (d < 8 || d % 8 || d > (1 << 20)) return fail(MSTAR_ERR_INVALID, "d must be a multiple of 8 in [8, 2^20]");
  return MSTAR_OK;
}

static Gemm plan(int B, int V, int d) {
  Gemm g{};
  g.B = B;
  g.V = V;
  g.d = d;
  g.N = (B + 15) & ~15;
  g.nkb = (d + BK - 1) / BK;
  g.ntiles = (V + BM - 1) / BM;
  g.stages = std::min(MAX_STAGES, SMEM_BUDGET / (A_BYTES + g.N * BK * 2));
  return g;
}

static int smem_bytes(const Gemm &g) { return g.stages * (A_BYTES + g.N * BK * 2) + 1024; }

// Workspace layout: the grid's ready flags (256-byte rounded), then one
// partial-tile slot [N][BM] fp32 per CTA; the grid is at most the SM count.
static int64_t flags_bytes(int grid) { return ((int64_t)grid * 4 + 255) / 256 * 256; }
static int64_t workspace_bytes(int B) {
  const int N = (B + 15) & ~15, G = sm_count();
  return flags_bytes(G) + (int64_t)G * N * BM * 4;
}

static int logits(const void *hidden, const void *weight, int B, int V, int d, void *out, int dtype, int64_t ld,
                  void *ws, int64_t ws_bytes, uint32_t *err, cudaStream_t st) {
  int rc = check_operands(hidden, weight, B, V, d);
  if (rc) return rc;
  if (!out) return fail(MSTAR_ERR_INVALID, "logits must not be NULL");
  if (dtype != MSTAR_DTYPE_F32 && dtype != MSTAR_DTYPE_BF16)
    return fail(MSTAR_ERR_INVALID, "dtype must be MSTAR_DTYPE_F32 or MSTAR_DTYPE_BF16");
  if (ld < V) return fail(MSTAR_ERR_INVALID, "ld must be >= V");
  Gemm g = plan(B, V, d);
  g.out = out;
  g.ld = ld;
  g.out_dtype = dtype;
  g.err = err;
  CUtensorMap tw, th;
  if ((rc = make_map(&tw, weight, V, d, BM))) return rc;
  if ((rc = make_map(&th, hidden, B, d, g.N))) return rc;
  const int smem = smem_bytes(g);
  cudaError_t e = cudaFuncSetAttribute(lmhead_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  const int G = sm_count();
  int grid = std::min(g.ntiles, G);
  if (ws) {
    if (reinterpret_cast<uintptr_t>(ws) & 255u) return fail(MSTAR_ERR_INVALID, "workspace must be 256-byte aligned");
    if (ws_bytes < workspace_bytes(B)) return fail(MSTAR_ERR_INVALID, "workspace too small");
    const int64_t units = (int64_t)g.ntiles * g.nkb;
    grid = (int)std::min<int64_t>(G, units);
    g.flags = static_cast<uint32_t *>(ws);
    g.ws = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + flags_bytes(G));
    e = cudaMemsetAsync(g.flags, 0, (size_t)grid * 4, st);
    if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  lmhead_gemm_kernel<<<grid, THREADS, smem, st>>>(tw, th, g);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MSTAR_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return MSTAR_OK;
}

// Projection scratch for callers that cannot allocate device memory: engines
// that hand all of HBM to their own pool at start-up (a raw cudaMalloc then
// fails or fragments the pool), code that runs while a stream is being
// captured in global mode (where cudaMalloc is not allowed), and native
// callers with no device allocator of their own.  The stream-K workspace of
// mstar_lmhead_logits_static lives here instead: a file-scope device array of
// STATIC_WS_BYTES (8 MiB), which every GPU that loads the library holds until
// the process exits.  All calls on a device share it and it keeps the last
// call's contents; each call clears the ready flags it relies on, and calls
// that overlap on the GPU (two streams, two threads) race on it.
constexpr int64_t STATIC_WS_BYTES = 8ll << 20;
static __device__ __align__(256) uint8_t g_static_ws[STATIC_WS_BYTES];

// Device address of g_static_ws on the current device, looked up once per
// device with that device current (g_static_ws itself is only a host-side
// stand-in for the symbol).  The lookup may load the module on the device,
// so the first call on a device should come before any stream capture.
static void *static_ws(int &rc) {
  static void *addr[kMaxDevices] = {};
  const int dev = current_device();
  std::lock_guard<std::mutex> g(g_dev_mu);
  if (!addr[dev]) {
    void *a = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&a, g_static_ws);
    if (e != cudaSuccess || !a) {
      rc = fail(MSTAR_ERR_CUDA, std::string("cudaGetSymbolAddress(static workspace): ") + cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = a;
  }
  rc = MSTAR_OK;
  return addr[dev];
}

static int logits_static(const void *hidden, const void *weight, int B, int V, int d, void *out, int dtype,
                         int64_t ld, uint32_t *err, cudaStream_t st) {
  if (B >= 1 && B <= MAX_N && workspace_bytes(B) > STATIC_WS_BYTES)
    return fail(MSTAR_ERR_INVALID, "B = " + std::to_string(B) + " needs " + std::to_string(workspace_bytes(B)) +
                                       " bytes of scratch; the static workspace holds " +
                                       std::to_string(STATIC_WS_BYTES) + " (at most 96 rows on 148 SMs)");
  int rc = check_operands(hidden, weight, B, V, d);
  if (rc) return rc;
  void *ws = static_ws(rc);
  if (rc) return rc;
  return logits(hidden, weight, B, V, d, out, dtype, ld, ws, STATIC_WS_BYTES, err, st);
}

}  // namespace lmh
