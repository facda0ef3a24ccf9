/*
 * ecah_sampler.h -- C ABI of the B200 token sampler (libecah_sampler.so).
 *
 * The library replaces the per-step sampling expression of the ecahLang
 * decode loop:
 *
 *   logits = logits / mask_penalty                      ecahlang/main.py:169
 *   logits = logits / temperature                       ecahlang/main.py:170
 *   idx = flashinfer.sampling.top_k_top_p_sampling_from_logits(
 *             logits, top_k=..., top_p=..., deterministic=True)
 *                                                       ecahlang/main.py:377-379
 *   (same expression at main.py:398-402, :486-491, :579-584)
 *
 * and the per-token repetition-penalty table update
 *
 *   manager.mask_penalty[slot, idx] /= rp  (or *= rp)   ecahlang/main.py:691-694
 *                                                       (also :519-522, :596-597)
 *
 * Every entry point takes plain device pointers and sizes, allocates nothing,
 * never synchronises the host and never traps; all work is enqueued on the
 * caller's stream, so the calls can be captured into a CUDA graph.  `stream`
 * is a cudaStream_t passed as void* so this header needs no CUDA include.
 * Status codes are returned; ecah_status_string() names them.
 */
#ifndef ECAH_SAMPLER_H
#define ECAH_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ECAH_SAMPLER_ABI_VERSION 2

#if defined(__GNUC__)
#define ECAH_API __attribute__((visibility("default")))
#else
#define ECAH_API
#endif

/* logits dtype: the model dtype of ecahlang/env.py (--torch_dtype) */
enum ecah_dtype { ECAH_DTYPE_F16 = 0, ECAH_DTYPE_BF16 = 1, ECAH_DTYPE_F32 = 2 };

enum ecah_status {
  ECAH_OK = 0,
  ECAH_ERR_NULL = 1,       /* a required pointer is NULL                         */
  ECAH_ERR_DTYPE = 2,      /* dtype is not one of enum ecah_dtype                */
  ECAH_ERR_SHAPE = 3,      /* batch/vocab/stride out of range (vocab too large)  */
  ECAH_ERR_WORKSPACE = 4,  /* workspace NULL or smaller than _workspace_bytes()  */
  ECAH_ERR_LAUNCH = 5,     /* the CUDA launch itself failed                      */
  ECAH_ERR_ABI = 6         /* args.abi_version does not match this library       */
};

/* flags */
#define ECAH_FLAG_FREQ_PRES 0x1u /* apply frequency/presence penalties (additive) */

/*
 * One sampler launch.  Row r of the batch samples one token id from
 * logits[r * row_stride + 0 .. vocab).  Per-row parameter arrays have `batch`
 * entries (stride 1).  Semantics per row (the reference's op order):
 *
 *   y  = D(x / m(c))              repetition penalty, D = model dtype rounding,
 *                                 m(c) = mask value after c updates (hist_mval),
 *                                 m(c+1) = D(m(c) * rep_factor)
 *   y' = D(y - (f*c + pi)) [c > 0]   only with ECAH_FLAG_FREQ_PRES (not in the reference);
 *                     the penalised logit stays in the model dtype D
 *   z  = y' / T                   float32; T <= 0 -> argmax (lowest index)
 *   top-k (k <= 0 or k >= vocab: off), ties with the k-th value kept
 *   softmax over the kept set, then top-p over it (p <= 0 or p >= 1: off)
 *   draw: smallest index whose inclusive cumulative mass (vocab order) > u * Z
 */
typedef struct ecah_sampler_args {
  int32_t abi_version;        /* = ECAH_SAMPLER_ABI_VERSION                      */
  int32_t dtype;              /* enum ecah_dtype                                  */
  int32_t batch;              /* B >= 0                                           */
  int32_t vocab;              /* V >= 1                                           */
  int64_t row_stride;         /* elements between rows, >= vocab                  */
  const void* logits;         /* [B, row_stride] model dtype                      */
  const float* temperature;   /* [B] (the reference's [B,1] buffer, contiguous)   */
  const int32_t* top_k;       /* [B]                                              */
  const float* top_p;         /* [B]                                              */
  /* penalties: NULL pointers mean "none" */
  const float* rep_factor;    /* [B] per-update mask multiplier: float32(1/rp) with the
                                 reciprocal taken in double if rp > 1, else float32(rp)
                                 -- what torch multiplies by for the reference's
                                 `mask /= rp` / `mask *= rp` on a CUDA tensor.  Used only
                                 to derive m(c) when hist_mval == NULL. */
  const float* freq_pen;      /* [B] f  (ECAH_FLAG_FREQ_PRES)                      */
  const float* pres_pen;      /* [B] pi (ECAH_FLAG_FREQ_PRES)                      */
  /* per-slot token histories (the sparse form of mask_penalty[slot, :]) */
  const int32_t* row_slot;    /* [B] slot of each row, -1 = no history; NULL = none */
  const int32_t* slot_len;    /* [S] live entries per slot                         */
  const int32_t* hist_tok;    /* [S, hist_cap] token ids (unique within a slot)    */
  const int32_t* hist_cnt;    /* [S, hist_cap] counts                              */
  const float* hist_mval;     /* [S, hist_cap] mask value m(c) in the model dtype,
                                 or NULL to derive it from rep_factor and the count */
  int32_t hist_cap;           /* entries per slot                                  */
  int32_t num_slots;          /* S; rows whose slot is outside [0, S) have no history */
  uint32_t flags;             /* ECAH_FLAG_*                                       */
  /* randomness: uniforms[B] in [0,1) if given, else Philox4x32-10 with
     state = {seed, offset}; the offset is advanced by 1 on the device after
     the launch (CUDA-graph safe). */
  const float* uniforms;
  uint64_t* philox_state;     /* [2] device memory                                 */
  int32_t* out;               /* [B] sampled token ids                             */
  /* optional outputs (NULL = skip; they cost an extra pass when requested) */
  float* row_stats;           /* [B, 4]: {y' threshold of the top-k set, y' threshold
                                 of the final set, M = max z, Z = kept mass}; the
                                 kept sets are {i : y'_i >= threshold}            */
  float* probs_out;           /* [B, vocab] renormalised probabilities of the final
                                 set (0 elsewhere); greedy rows get a one-hot row */
  void* workspace;            /* >= ecah_sampler_workspace_bytes(B, vocab, dtype) for
                                 some B >= batch, zero-filled once before first use.
                                 Its first 4096 bytes hold counters that every launch
                                 leaves at zero; the rest is scratch.               */
  size_t workspace_bytes;
  /* Row gather (prefill): row r samples logits row row_index[r] of a
     [logit_rows, row_stride] buffer, e.g. the last token of each request,
     append_indptr[1:] - 1 (ecahlang/main.py:476), with no [B, V] copy.
     NULL = row r reads row r (logit_rows is then ignored).  Entries outside
     [0, logit_rows) are clamped into it; callers check them.  Penalty slots,
     parameters and outputs stay indexed by r. */
  const int32_t* row_index;   /* [B] device                                        */
  int32_t logit_rows;         /* rows of the logits buffer (>= 1 with row_index)   */
} ecah_sampler_args;

ECAH_API int ecah_sampler_abi_version(void);
ECAH_API const char* ecah_status_string(int status);

/* Workspace for launches of up to `batch` rows of this vocabulary and dtype
 * on the current device (small batches split rows over several CTAs, which
 * needs room that depends on the device's SM count).  New entry point:
 * FlashInfer's sampling ops allocate their row-state buffers themselves
 * (called from ecahlang/main.py:377-379); here the caller owns them. */
ECAH_API size_t ecah_sampler_workspace_bytes(int32_t batch, int32_t vocab, int32_t dtype);

/* Sample one token per row.  Replaces the two divides and
 * flashinfer.sampling.top_k_top_p_sampling_from_logits at
 * ecahlang/main.py:169-170, :377-379, :398-402, :486-491, :579-584. */
ECAH_API int ecah_sampler_launch(const ecah_sampler_args* args, void* stream);

/* Record the sampled ids in the slot histories: for each row with
 * row_slot[r] in [0, num_slots), the entry of token ids[r] gets count += 1
 * and m <- D(m * rep_factor[r]) (a new entry starts at m = 1, count = 0
 * before the update; rep_factor as in ecah_sampler_args, NULL = 1).  Replaces the per-request
 * `mask_penalty[slot, idx] /= rp` launches of ecahlang/main.py:691-694
 * (also :519-522, :596-597); a full slot sets overflow[slot] = 1 and drops
 * the token.  `overflow` may be NULL. */
ECAH_API int ecah_hist_update(const int32_t* ids, int32_t batch, const int32_t* row_slot,
                              const float* rep_factor, int32_t* slot_len, int32_t* hist_tok,
                              int32_t* hist_cnt, float* hist_mval, int32_t hist_cap,
                              int32_t num_slots, int32_t dtype, int32_t* overflow,
                              void* stream);

/* The per-row uniforms the sampler draws with when args.uniforms == NULL
 * (same Philox mapping), written to out[B]; advance != 0 also bumps the
 * offset.  Stands in for the torch-generator seed/offset read of
 * FlashInfer's sampling ops (called from ecahlang/main.py:377-379). */
ECAH_API int ecah_philox_uniforms(uint64_t* philox_state, int32_t batch, float* out,
                         int32_t advance, void* stream);

/* ecah_sampler_launch without a caller workspace, for callers that cannot
 * allocate device memory at sampling time (a runtime that owns all device
 * memory through its own pool, an FFI caller with no CUDA allocator).  No
 * counterpart in the reference: FlashInfer's sampler allocates its own state.
 * Scratch is a fixed array of ecah_sampler_noalloc_scratch_bytes() bytes in
 * the library's device memory, held on every GPU that loads the library until
 * exit.  That is the least any launch accepts, so every shape runs the
 * cluster kernel (slower than ecah_sampler_launch with a full workspace);
 * shapes the cluster kernel cannot take get ECAH_ERR_SHAPE.  Every call looks
 * up the array's address on the current device; the first call on a device
 * may load the module, so make it outside stream capture.  Calls share the
 * array, so calls overlapping on the GPU race.  args->workspace and
 * args->workspace_bytes are ignored. */
ECAH_API int ecah_sampler_launch_noalloc(const ecah_sampler_args* args, void* stream);
ECAH_API size_t ecah_sampler_noalloc_scratch_bytes(void);

/* Diagnostic; no counterpart in the reference.  For each of the n_temperature
 * device temperatures T[t], compares y / T as the kernels compute it for
 * softmax masses (reciprocal plus one correction step) with the IEEE float32
 * quotient torch computes for `logits / temperature` (ecahlang/main.py:170),
 * over every input y of `dtype` (every fp16 or bf16 bit pattern, or every
 * float32 bit pattern).  counts (device, 3 * n_temperature entries), over
 * finite inputs whose IEEE quotient is a normal float32: counts[3t] = more
 * than one unit in the last place apart, counts[3t+1] = exactly one unit
 * apart; counts[3t+2] = the rest (zero signs, subnormal quotients, non-finite
 * inputs).  A float32 sweep takes a few milliseconds per temperature. */
ECAH_API int ecah_quotient_mismatches(int32_t dtype, const float* temperature, int32_t n_temperature,
                                      unsigned long long* counts, void* stream);

/*
 * Vocab-parallel sampling (fp16/bf16 logits).  Each of `world` ranks holds
 * columns [vocab_offset, vocab_offset + vocab_local) of the [batch, vocab]
 * logits.  ecah_vp_local writes, per row, every local entry whose key is >=
 * the slice's k-th largest key (ties included; k = top_k, 1 for greedy rows)
 * in vocab order as (key << 32 | global id), at most cand_cap of them, and
 * their count (rows whose k exceeds cand_cap get no list and count = k).
 * The caller all-gathers cand/cand_count over the ranks (rank order) into
 * all_cand/all_count; ecah_vp_merge then draws the same token on every rank
 * (the same uniforms / Philox state on every rank).  Rows need
 * 1 <= top_k <= cand_cap (or T <= 0); rows with top-k off, or whose lists
 * were truncated (count > cand_cap), get out = -1 here; those without top-k
 * are then drawn by ecah_vp_dist_pass.  Replaces the whole-row FlashInfer call of
 * ecahlang/main.py:377-379 when the LM head is split by vocabulary (ecahLang
 * itself runs on one GPU, ecahlang/env.py:112).
 */
typedef struct ecah_vp_args {
  int32_t abi_version;        /* = ECAH_SAMPLER_ABI_VERSION                      */
  int32_t dtype;              /* ECAH_DTYPE_F16 or ECAH_DTYPE_BF16               */
  int32_t batch;
  int32_t vocab;              /* full vocabulary                                 */
  int32_t vocab_offset;       /* this rank's first column                        */
  int32_t vocab_local;        /* this rank's columns, 1 .. 524288                */
  int64_t row_stride;         /* elements between rows of the local slice        */
  const void* logits;         /* [batch, row_stride] local slice                 */
  const float* temperature;   /* [batch]                                         */
  const int32_t* top_k;       /* [batch]                                         */
  const float* top_p;         /* [batch]                                         */
  const float* rep_factor;    /* as in ecah_sampler_args; history ids are global */
  const int32_t* row_slot;
  const int32_t* slot_len;
  const int32_t* hist_tok;
  const int32_t* hist_cnt;
  const float* hist_mval;
  int32_t hist_cap;
  int32_t num_slots;
  int32_t cand_cap;           /* candidates per row and rank, 1 .. 2048 / world  */
  uint64_t* cand;             /* [batch, cand_cap] written by ecah_vp_local      */
  int32_t* cand_count;        /* [batch] written by ecah_vp_local                */
  int32_t world;              /* ranks, 1 .. 64                                  */
  const uint64_t* all_cand;   /* [world, batch, cand_cap] gathered lists          */
  const int32_t* all_count;   /* [world, batch] gathered counts                   */
  const float* uniforms;      /* [batch], or NULL: Philox from philox_state       */
  uint64_t* philox_state;     /* [2], advanced by 1 after the merge               */
  int32_t* out;               /* [batch] sampled ids (the same on every rank)     */
  float* row_stats;           /* [batch, 4] optional, as in ecah_sampler_args     */
  void* workspace;            /* >= 256 bytes, zero-filled once                   */
  size_t workspace_bytes;
} ecah_vp_args;

ECAH_API int ecah_vp_local(const ecah_vp_args* args, void* stream);
ECAH_API int ecah_vp_merge(const ecah_vp_args* args, void* stream);

/* Rows without top-k (T > 0 and top_k <= 0 or >= vocab: the reference's
 * default request, ecahlang/main.py:643, and top-p-only rows), whose kept set
 * the candidate lists cannot hold: the exact distributed sampler, run over
 * this rank's slice for the `nrows` batch rows listed in `rows` (device
 * int32).  Listed rows that have a top-k or T <= 0 are skipped (their ids are
 * left as they are), so a caller may list every row.  `state` is a device
 * float [nrows, 8] per-row state.  pass selects one step:
 *   1..5   (slice passes, in = state (unused by pass 1), out = the pass's
 *           outputs, float [nrows, w]):
 *     1  w = 3: {z of the slice max, lowest global id holding it, slice mass}
 *     2  w = 256: masses (relative to the row max) per high byte of the key
 *     3  w = 257: masses per low key byte inside the chosen high byte, and
 *        [256] the mass above it
 *     4  w = 1: the slice's kept mass (keys >= the top-p threshold's tie
 *        floor and the zero-mass cut)
 *     5  w = 1 (int32): on the rank that owns the draw, the lowest global id
 *        whose cumulative kept mass in vocab order exceeds its target; -1
 *        elsewhere
 *   11..15 (combine after pass 1..5, in = the combined outputs, out = state):
 *     11  in = pass 1 all-gathered [world, nrows, 3] (rank order)
 *     12  in = pass 2 summed over the ranks [nrows, 256]
 *     13  in = pass 3 summed over the ranks [nrows, 257]
 *     14  in = pass 4 all-gathered [world, nrows]; the uniform is
 *         uniforms[row], else the Philox uniform of the current state
 *     15  in = pass 5 max over the ranks [nrows] (int32): writes out[row]
 *         (-1 for a row with a NaN logit).
 * So one step runs 1, all-gather, 11, 2, all-reduce, 12, 3, all-reduce, 13,
 * 4, all-gather, 14, 5, all-reduce (max), 15.  Combine 11 already chooses
 * the owning rank of a row without top-p (its kept set is every entry above
 * the zero-mass cut), and passes 2-4 skip such rows: when no listed row has
 * 0 < top_p < 1 the step is 1, all-gather, 11, 5, all-reduce (max), 15.  Keys are the
 * order-preserving 16-bit keys of the penalised logits; the top-p threshold
 * is the reference's (the largest z whose mass from the top reaches
 * top_p * Z).  New entry point: the reference runs on one GPU. */
ECAH_API int ecah_vp_dist_pass(const ecah_vp_args* args, int32_t rank, int32_t pass, const int32_t* rows,
                               int32_t nrows, const void* in, void* out, void* stream);

/*
 * The whole vocab-parallel step in one kernel per rank, with the exchange
 * over NVLink peer memory instead of an all-gather.  Each rank owns an
 * exchange buffer of ecah_vp_exchange_bytes(max_batch, world, cand_cap) bytes
 * (ecah_vp_ipc_alloc: zero-filled, with a CUDA IPC handle) and maps every
 * other rank's (ecah_vp_ipc_open).  Per row, the kernel stores its list and
 * count into its slot of every rank's buffer, sets the row's flag there, waits
 * for every rank's flag in its own buffer (at most timeout_us per wait), then
 * merges and draws as ecah_vp_merge does.  Every rank launches every step with
 * the same batch, parameters and uniforms (or Philox state).  A wait that runs
 * out sets the error word (int32 at byte 8 of this rank's buffer); that row
 * and the rest of the step get out = -1.  args->cand, cand_count, all_cand,
 * all_count, workspace are not used.  The step counter lives in the buffer,
 * so the launch can be captured in a CUDA graph.  Ranks on one GPU are not
 * supported (their kernels would wait on each other).
 */
typedef struct ecah_vp_peers {
  int32_t rank;               /* this rank, 0 .. world-1                          */
  int32_t max_batch;          /* rows the exchange buffers were sized for         */
  void* const* base;          /* device array [world]: every rank's exchange
                                 buffer as mapped in this process (own at rank)  */
  uint32_t timeout_us;        /* per wait on another rank's row                   */
} ecah_vp_peers;

ECAH_API size_t ecah_vp_exchange_bytes(int32_t max_batch, int32_t world, int32_t cand_cap);
ECAH_API int ecah_vp_step(const ecah_vp_args* args, const ecah_vp_peers* peers, void* stream);
/* CUDA IPC helpers for the exchange buffers (handle: 64 bytes). */
ECAH_API int ecah_vp_ipc_alloc(size_t bytes, void** ptr, void* handle);
ECAH_API int ecah_vp_ipc_open(const void* handle, void** ptr);
ECAH_API int ecah_vp_ipc_close(void* ptr);
ECAH_API int ecah_vp_ipc_free(void* ptr);
/* Recovery after a step whose wait ran out (error word set), or after a rank
 * skipped a step: writes this rank's exchange-buffer header to {epoch, 0
 * finished rows, error 0} on `stream`.  The error word is sticky until then:
 * every later step of this rank returns -1 for every row.  Call it on every
 * rank with the same epoch -- the largest step counter over the ranks (the
 * uint32 at byte 0 of each buffer) -- after a host barrier with no step in
 * flight on any rank, then barrier again before the next step.  No
 * counterpart in the reference, which runs on one GPU. */
ECAH_API int ecah_vp_reset(void* own_buffer, uint32_t epoch, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ECAH_SAMPLER_H */
