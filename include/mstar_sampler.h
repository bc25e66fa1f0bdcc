/*
 * mstar_sampler.h -- C ABI of the B200 batched token sampler.
 *
 * Plain pointers and sizes only; every pointer below is a DEVICE pointer on
 * the current CUDA device unless stated otherwise.  All calls are
 * asynchronous on `stream` (a cudaStream_t passed as void*), allocate
 * nothing, never synchronise, and are therefore legal inside CUDA-graph
 * capture.  Argument validation happens on the host before any launch; a
 * non-zero return means nothing was launched.
 *
 * Reference interfaces these entry points replace (npuichigo/mstar-rs; the
 * sampler itself lives in the external `mstar.utils.sampling` package):
 *   mstar_sampler_step      <- CudaGraphableSampler.sample(rids, logits, apply_penalty=True)
 *                              python/mstar_rs/models/orpheus.py:350, :496;
 *                              python/mstar_rs/models/qwen3_omni.py:518
 *                              (and the eager Sampler.sample, orpheus.py:517,
 *                              qwen3_omni.py:483), plus the in-graph seen-mask
 *                              update synced back at orpheus.py:426 and the
 *                              offset_buf advance saved/restored at orpheus.py:353-359
 *   mstar_sampler_tp_local  <- the vocab-parallel half of the TP sampler whose
 *   mstar_sampler_tp_merge     tp_group keeps Thinker ranks in agreement
 *                              (python/mstar_rs/models/qwen3_omni.py:401-404, :408, :431)
 *   mstar_sampler_plan      <- launch planning behind SamplerBuffers.allocate
 *                              (orpheus.py:101-103, qwen3_omni.py:431, :987-989)
 */
#ifndef MSTAR_SAMPLER_H_
#define MSTAR_SAMPLER_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MSTAR_SAMPLER_ABI_VERSION 2

/* logits dtypes */
#define MSTAR_DTYPE_F32 0
#define MSTAR_DTYPE_BF16 1

/* flags */
#define MSTAR_FLAG_UPDATE_HISTORY 0x1u /* append the sampled id to hist_ids/hist_len */
#define MSTAR_FLAG_UPDATE_SEEN 0x2u    /* set the sampled id's bit in seen_bits */
#define MSTAR_FLAG_ADVANCE_OFFSET 0x4u /* offset[slot] += 1 after the draw */
#define MSTAR_FLAG_FORCE_GENERAL 0x8u  /* testing: take the multi-round selection path */
#define MSTAR_FLAG_TEST_WITHHOLD 0x10u /* testing: leave each CTA's last bulk copy unissued, so its
                                          bounded wait (2 ms) runs out: MSTAR_STATUS_TIMEOUT */

/* per-row status bits written to out_status */
#define MSTAR_STATUS_EMPTY 0x1u        /* no token had positive weight; id 0 returned */
#define MSTAR_STATUS_GENERAL 0x2u      /* row took the multi-round selection path */
#define MSTAR_STATUS_SPECIAL_OVERFLOW 0x4u /* more penalised/biased ids than the table holds */
#define MSTAR_STATUS_TP_OVERFLOW 0x8u  /* TP: a shard's candidate set exceeded tp_cap */
#define MSTAR_STATUS_TIMEOUT 0x10u     /* a bounded wait (2 ms) on a bulk copy gave up; the id is not valid */
#define MSTAR_STATUS_STOP 0x20u        /* the sampled id is one of the slot's stop ids */
#define MSTAR_STATUS_BAD_RECORD 0x40u  /* TP merge: a record entry held an id >= V_global (left out) */

/* return codes */
#define MSTAR_OK 0
#define MSTAR_ERR_INVALID 1
#define MSTAR_ERR_UNSUPPORTED 2
#define MSTAR_ERR_CUDA 3

typedef struct mstar_sampler_params {
  /* logits [B, ld], row r holds columns [0, V) of the vocabulary shard that
   * starts at global id `vocab_offset` (0 without tensor parallelism). */
  const void *logits;
  int32_t dtype;
  int32_t B;
  int32_t V;
  int32_t num_slots;         /* rows of every per-slot array below */
  int64_t ld;                /* row stride in elements */
  int64_t vocab_offset;
  const int32_t *slot_idx;   /* [B] or NULL (row r uses slot r); <0 = padding row */

  /* per-slot sampling parameters, [num_slots] each; NULL = default
   * (temperature 1, top_k 0, top_p 1, min_p 0, rep 1, presence 0, frequency 0) */
  const float *temperature;
  const int32_t *top_k;
  const float *top_p;
  const float *min_p;
  const float *rep_pen;
  const float *pres_pen;
  const float *freq_pen;

  /* penalty input, at most one of:
   *   token history  hist_ids [num_slots, H] (global ids, ring of the last H
   *                  generated tokens) + hist_len [num_slots]
   *   seen bitmask   seen_bits [num_slots, seen_words] (bit g&31 of word g>>5)
   * Any number of bits may be set.  seen_cap is not read (kept so the layout
   * of this struct stays the same). */
  int32_t *hist_ids;
  int32_t *hist_len;
  int32_t H;
  int32_t seen_cap;
  uint32_t *seen_bits;
  int64_t seen_words;

  /* logit bias [num_slots, NB]; id < 0 marks an unused entry */
  const int32_t *bias_ids;
  const float *bias_vals;
  int32_t NB;
  int32_t pad0;

  /* allowed-token bitmask [num_slots, allowed_words] or NULL (all allowed) */
  const uint32_t *allowed_bits;
  int64_t allowed_words;

  /* randomness: uniforms [B] in [0,1) if non-NULL, else Philox4x32-10 keyed
   * by seed[slot] at counter offset[slot] */
  const float *uniforms;
  const uint64_t *seed;
  uint64_t *offset;

  /* outputs */
  int64_t *out_ids;          /* [B] global token ids (or NULL) */
  int32_t *out_ids32;        /* [B] (or NULL) */
  int32_t *out_status;       /* [B] (or NULL) */
  /* debug / verification outputs, [B, V] each, or NULL */
  float *out_x;              /* processed logits */
  uint8_t *out_kept;         /* kept-set membership */
  float *out_probs;          /* normalised probabilities over the kept set */

  uint32_t flags;
  int32_t cluster_size;      /* CTAs per row; 0 = automatic */

  /* stop tokens (replaces the host-side `token == stop_token_id` test after
   * every step, python/mstar_rs/models/orpheus.py:428-432, :518-519):
   * stop_ids [num_slots, NS] global ids, id < 0 marks an unused entry, or
   * NULL.  A row whose sampled id is one of its slot's stop ids gets
   * MSTAR_STATUS_STOP in out_status and, when stop_flags [num_slots] is
   * non-NULL, stop_flags[slot] = 1 (set only; the caller clears it). */
  const int32_t *stop_ids;
  int32_t NS;
  int32_t pad1;
  int32_t *stop_flags;
} mstar_sampler_params_t;

/* Library ABI version (MSTAR_SAMPLER_ABI_VERSION). */
int mstar_sampler_abi_version(void);

/* Human-readable text for the last host-side error in this thread. */
const char *mstar_sampler_last_error(void);

/* Dynamic shared memory per CTA and CTAs per row the step would use for
 * these parameters (no launch). Returns MSTAR_OK or an error code. */
int mstar_sampler_plan(const mstar_sampler_params_t *p, int32_t *cluster_size,
                       int64_t *smem_bytes);

/* One sampling step for B rows: logits -> token ids, with per-slot state
 * (RNG offset, history / seen bits) advanced on the device. */
int mstar_sampler_step(const mstar_sampler_params_t *p, void *stream);

/* Tensor-parallel sampling over a vocabulary shard.
 * tp_local: writes this shard's candidate record for every row into
 *   send [B, rec_words] (uint32 words; rec_words = mstar_sampler_tp_record_words(tp_cap)).
 * tp_merge: reads the all-gathered records recv [tp_world, B, rec_words] and
 *   produces the same ids and state updates on every rank.  p->V / vocab_offset
 *   describe this rank's shard; V_global is the full vocabulary. */
int32_t mstar_sampler_tp_record_words(int32_t tp_cap);
int mstar_sampler_tp_local(const mstar_sampler_params_t *p, int32_t tp_cap, uint32_t *send,
                           void *stream);
int mstar_sampler_tp_merge(const mstar_sampler_params_t *p, int32_t tp_cap, int32_t tp_world,
                           int64_t V_global, const uint32_t *recv, void *stream);

/* Two-round tensor-parallel sampling, for rows without top_k (or with one
 * above tp_cap): the reference's Thinker samples with top_k 0 whenever a
 * temperature is given (python/mstar_rs/models/qwen3_omni.py:440-443).
 *   1. tp_local2: as tp_local, but such a row sends the first tp_cap members
 *      of its shard A set (record word 3, bit 0: possibly partial) and
 *      leaves the shard's final values in xbuf [B, V] (f32).
 *   2. all-gather the records; tp_merge1 on every rank: rows with no partial
 *      shard are decided as by tp_merge; the others are deferred, and pend
 *      [B, 2] (uint32: flag, bits of the row max M) records them.
 *   3. tp_mass: the shard's exact A mass against M for every deferred row
 *      into send2 [B, 2] (uint32 pairs, a little-endian u64 each; 0 for the
 *      rest).
 *   4. all-gather send2 into recv2 [tp_world, B, 2]; tp_merge2 on every rank
 *      decides the deferred rows exactly when their kept set (top_p) or draw
 *      point (no top_p) lies among the members every shard sent, and flags
 *      the rest MSTAR_STATUS_TP_OVERFLOW (id: the row's leading member).
 * Every rank gets the same ids and state updates.  tp_world <= 16. */
int mstar_sampler_tp_local2(const mstar_sampler_params_t *p, int32_t tp_cap, uint32_t *send,
                            float *xbuf, void *stream);
int mstar_sampler_tp_merge1(const mstar_sampler_params_t *p, int32_t tp_cap, int32_t tp_world,
                            int64_t V_global, const uint32_t *recv, uint32_t *pend, void *stream);
int mstar_sampler_tp_mass(const mstar_sampler_params_t *p, const float *xbuf, const uint32_t *pend,
                          uint32_t *send2, void *stream);
int mstar_sampler_tp_merge2(const mstar_sampler_params_t *p, int32_t tp_cap, int32_t tp_world,
                            int64_t V_global, const uint32_t *recv, const uint32_t *recv2,
                            const uint32_t *pend, void *stream);

/* State updates for ids chosen elsewhere: for every row r of [0, p->B)
 * whose slot (slot_idx[r], or r) is >= 0 and whose id ids[r] lies in
 * [vocab_offset, vocab_offset + V): append the id to the slot's history ring
 * (MSTAR_FLAG_UPDATE_HISTORY), set its seen bit (MSTAR_FLAG_UPDATE_SEEN),
 * advance the slot's RNG offset (MSTAR_FLAG_ADVANCE_OFFSET) and flag a stop
 * id (stop_ids / stop_flags), exactly as a step that sampled those ids would.
 * Used after the tensor-parallel broadcast of rank 0's ids (the reference's
 * tp_group broadcast, python/mstar_rs/models/qwen3_omni.py:401-404), so the
 * per-slot state of every rank takes the same ids; also for ids an engine
 * appends itself (SeenTokenMask.add_tokens, orpheus.py:500).  Reads only the
 * fields named here; logits may be NULL.  ids: [B] int64 (device). */
int mstar_sampler_commit(const mstar_sampler_params_t *p, const int64_t *ids, void *stream);

/* LM-head projection on the tensor cores: logits[b * ld + v] = sum_k
 * hidden[b * d + k] * weight[v * d + k] for b < B, v < V; hidden [B, d] and
 * weight [V, d] bf16 row-major (a Linear's weight), fp32 accumulation,
 * stored as dtype (MSTAR_DTYPE_F32, or MSTAR_DTYPE_BF16 rounded to nearest
 * even).  Replaces the `self.lm_head(hidden)` that precedes each sampler
 * call (python/mstar_rs/models/orpheus.py:349, qwen3_omni.py:517).
 * B <= 256, d a multiple of 8, both pointers 16-byte aligned.
 * workspace: NULL, or device scratch of at least
 * mstar_lmhead_workspace_bytes(B) bytes (256-byte aligned; its contents
 * need not be preserved between calls, and calls that share it must not
 * overlap on the GPU).  With it every SM gets an equal share of the weight
 * stream (split vocabulary tiles are summed through it); without it the
 * shares are whole 128-id tiles.  status: NULL or a device word that gets
 * bit 1 if a bounded in-kernel wait ran out. */
int64_t mstar_lmhead_workspace_bytes(int32_t B);
int mstar_lmhead_logits(const void *hidden, const void *weight, int32_t B, int32_t V, int32_t d,
                        void *logits, int32_t dtype, int64_t ld, void *workspace,
                        int64_t workspace_bytes, uint32_t *status, void *stream);

/* mstar_lmhead_logits for callers that cannot allocate device memory: no
 * counterpart in the reference.  Engines that give all of HBM to their own
 * pool at start-up (a raw cudaMalloc then fails or fragments it), code that
 * runs during a global-mode stream capture (where cudaMalloc is not
 * allowed) and native callers without a device allocator pass only inputs
 * and outputs; the projection's scratch is a static device array of 8 MiB
 * inside the library, held on every GPU that loads the library until the
 * process exits.  The call allocates and frees nothing.  B is limited to
 * what fits that array (96 rows on a 148-SM GPU); larger B is refused with
 * MSTAR_ERR_INVALID.  The first call on a device looks the array's address
 * up (which may load the library's device code there): make it before any
 * stream capture.  All calls on a device share the array and leave their
 * contents in it (each call clears what it needs cleared); calls that
 * overlap on the GPU, from two streams or two threads, race on it. */
int mstar_lmhead_logits_static(const void *hidden, const void *weight, int32_t B, int32_t V,
                               int32_t d, void *logits, int32_t dtype, int64_t ld, uint32_t *status,
                               void *stream);

/* Projection and sampling in one call: mstar_lmhead_logits into p->logits
 * (which must be writable, [B, ld] of p->dtype, weight [p->V, d] being this
 * shard's rows), then mstar_sampler_step on it as a programmatic dependent
 * launch.  The logits are stored with an L2 evict-last policy and the
 * weight stream is read evict-first, so the step's logits are read back
 * from L2 rather than from HBM.  Results are those of the two calls made in
 * turn.  workspace, status: as for mstar_lmhead_logits. */
int mstar_sampler_lmhead_step(const mstar_sampler_params_t *p, const void *hidden, const void *weight,
                              int32_t d, void *workspace, int64_t workspace_bytes, uint32_t *status,
                              void *stream);

/* The sampler's Philox4x32-10 uniform for (seed, offset), computed on the
 * host; lets callers reproduce a draw without a device. */
float mstar_sampler_philox_uniform(uint64_t seed, uint64_t offset);

#ifdef __cplusplus
}
#endif

#endif /* MSTAR_SAMPLER_H_ */
