// Streaming token sampler for sm_100a in two launches, no clusters and no CTA
// that waits on another.
//
// stream_scan_kernel (persistent, about four 256-thread CTAs per SM) walks the
// (row, 8192-entry chunk) units with a two-buffer cp.async pipeline: every
// chunk is read from HBM once, the repetition-penalty patch of the row's slot
// history is applied, the logits become order-preserving 16-bit keys, and the
// chunk leaves a small summary in the workspace:
//   - the chunk max key and the lowest index holding it (greedy rows);
//   - rows with top-k or top-p: every entry whose key lies in the chunk's own
//     top N (N = k, or kSDense for top-p-only rows) -- the "candidates" --
//     found from a 64-bin histogram of the 2048 keys below the chunk max and
//     written in vocab order as (key << 16 | offset in chunk);
//   - rows without top-k: the softmax mass of the chunk relative to its own
//     max, sum exp(z - m_c), rescaled once the row max is known.
// stream_finish_kernel (one CTA per row) then finishes each row: row max M,
// the top-k and top-p thresholds from an exact per-key
// histogram of the candidates, the kept mass Z, then the inverse-CDF draw
// over the candidates in vocab order.  Every entry whose key is >= F (the
// highest candidate floor of the row's chunks) is a candidate, so the result
// is exact whenever both thresholds lie at or above F; when they do not, the
// finishing CTA re-reads the row (from L2) and runs a two-digit radix select.
// The launch boundary orders the summaries before their readers: no fences,
// counters or waits between CTAs.
// Rows without top-k and top-p draw from the per-chunk masses and re-read the
// one chunk that holds u*Z.
//
// Op order and tie rules are those of the cluster kernel (sampler_kernel.cuh),
// whose helpers (masses, tie floors, zero-mass cut) this kernel shares.
#pragma once

#include "sampler_kernel.cuh"

namespace ecah {

constexpr int kSCH = 8192;                 // vocab entries per chunk
constexpr int kSVecs = kSCH / 8;           // 16-byte vectors per chunk
constexpr int kSPerT = kSCH / kThreads;    // entries per thread (contiguous)
constexpr int kSWords = kSPerT / 2;        // packed key words per thread
constexpr int kSWin = 2048;                // keys below the chunk max that can hold candidates
constexpr int kSBins = kSWin / 32;         // candidate-window bins of 32 keys
constexpr int kSCap = 1024;                // candidates stored per chunk
constexpr int kSDense = 384;               // candidates aimed for per chunk, top-p-only rows
constexpr int kSMaxChunks = 64;
constexpr int kSStage = kSCH / 2;          // candidate entries one chunk buffer holds
constexpr unsigned kNoFloor = 0x10000u;    // above every 16-bit key
constexpr unsigned kSentinel = 0xFFFFu;    // list padding: offset field 0xFFFF
constexpr float kGenFx = 1048576.0f;       // fixed-point scale of fallback level-0 masses (2^20)
constexpr float kGenFxInv = 1.0f / 1048576.0f;

struct ChunkSum {
  unsigned lmax;   // chunk max key
  unsigned floor;  // every entry with key >= floor is a candidate (kNoFloor: none)
  int ncand;       // candidates written
  int first;       // lowest row index holding lmax
  float mref;      // value(lmax) / T
  float sref;      // sum of exp(z - mref) over the chunk (rows without top-k)
  unsigned pad0, pad1;
};

struct RowFin {    // what the probability kernel needs of a finished row
  float M, Z;
  unsigned kdraw;
  int mode;        // 0: mass / Z over keys >= kdraw; 1: one-hot at idx; 2: all zero
  int idx;
  int pad0, pad1, pad2;
};

struct SSmem {
  uint4 raw[2][kSVecs];           // two chunk buffers (pipeline) / staged candidate lists
  unsigned hist[kSWin];           // lane-private window bins / finisher histograms
  unsigned binc[kSBins];
  unsigned uw[kWarps];
  int iw[kWarps];
  float fw[kWarps];
  unsigned lm[kSMaxChunks];
  int nc[kSMaxChunks];
  int fi[kSMaxChunks];
  int pre[kSMaxChunks + 1];       // staged offsets of the chunk lists (entries)
  float mr[kSMaxChunks];
  float sr[kSMaxChunks];
  float ps[kSMaxChunks];
  float ct[kSMaxChunks];
  float l0f[64];
  int ib[16];
  float fb[16];
};

// ------------------------------------------------------------ block helpers
// All of them must be reached by every thread of the CTA.
__device__ __forceinline__ unsigned sblock_max(unsigned v, unsigned* uw) {
  v = __reduce_max_sync(0xFFFFFFFFu, v);
  if ((threadIdx.x & 31) == 0) uw[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned m = 0u;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) m = max(m, uw[w]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ int sblock_min(int v, int* iw) {
  v = __reduce_min_sync(0xFFFFFFFFu, v);
  if ((threadIdx.x & 31) == 0) iw[threadIdx.x >> 5] = v;
  __syncthreads();
  int m = INT_MAX;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) m = min(m, iw[w]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ int sblock_maxi(int v, int* iw) {
  v = __reduce_max_sync(0xFFFFFFFFu, v);
  if ((threadIdx.x & 31) == 0) iw[threadIdx.x >> 5] = v;
  __syncthreads();
  int m = INT_MIN;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) m = max(m, iw[w]);
  __syncthreads();
  return m;
}

// sum in a fixed order (deterministic)
__device__ __forceinline__ float sblock_sum(float v, float* fw) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) fw[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) t += fw[w];
  __syncthreads();
  return t;
}

__device__ __forceinline__ int sblock_excl_scan(int v, int* iw, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) iw[warp] = incl;
  __syncthreads();
  int base = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const int t = iw[w];
    if (w < warp) base += t;
    tot += t;
  }
  __syncthreads();
  *total = tot;
  return base + incl - v;
}

__device__ __forceinline__ float sblock_excl_scanf(float v, float* fw, float* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) fw[warp] = incl;
  __syncthreads();
  float base = 0.f, tot = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const float t = fw[w];
    if (w < warp) base += t;
    tot += t;
  }
  __syncthreads();
  *total = tot;
  return base + (incl - v);
}

// Same selection rule as warp_select (first position whose running total
// reaches `target`, else the last non-zero position), reading the histogram
// from shared memory twice instead of holding it in registers.
template <typename T, int NB, bool DESC>
__device__ void warp_select_seq(const T* hist, T target, int* out_bin, T* out_above) {
  constexpr int PER = NB / 32;
  const int lane = threadIdx.x & 31;
  T s = 0;
  for (int j = 0; j < PER; ++j) {
    const int pos = lane * PER + j;
    s += hist[DESC ? NB - 1 - pos : pos];
  }
  T incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  T excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
  if (lane == 0) excl = 0;
  const unsigned hit = __ballot_sync(0xFFFFFFFFu, incl >= target && s > 0);
  int pos = -1;
  T above = 0;
  int L;
  if (hit) {
    L = __ffs(hit) - 1;
    if (lane == L) {
      T acc = excl, acc_last = 0;
      int last_nz = -1;
      for (int j = 0; j < PER; ++j) {
        const int p = lane * PER + j;
        const T v = hist[DESC ? NB - 1 - p : p];
        if (v > 0) { last_nz = j; acc_last = acc; }
        if (v > 0 && acc + v >= target) { pos = p; above = acc; break; }
        acc += v;
      }
      if (pos < 0) { pos = lane * PER + (last_nz >= 0 ? last_nz : PER - 1); above = acc_last; }
    }
  } else {
    const unsigned nz = __ballot_sync(0xFFFFFFFFu, s > 0);
    L = nz ? 31 - __clz(nz) : 31;
    if (lane == L) {
      int jb = PER - 1;
      T acc = excl, acc_jb = excl;
      for (int j = 0; j < PER; ++j) {
        const int p = lane * PER + j;
        const T v = hist[DESC ? NB - 1 - p : p];
        if (v > 0) { jb = j; acc_jb = acc; }
        acc += v;
      }
      pos = lane * PER + jb;
      above = acc_jb;
    }
  }
  pos = __shfl_sync(0xFFFFFFFFu, pos, L);
  above = __shfl_sync(0xFFFFFFFFu, above, L);
  if (lane == 0) { *out_bin = DESC ? NB - 1 - pos : pos; *out_above = above; }
}

// key j (0..31) of a thread's packed key words
#define ECAH_SKEY(w, j) ((((j) & 1) != 0) ? ((w)[(j) >> 1] >> 16) : ((w)[(j) >> 1] & 0xFFFFu))

// ----------------------------------------------------------- chunk staging
// Chunk c of `row` into `buf`: raw logits of the model dtype with the
// repetition-penalty divide applied to the slot's history tokens; entries
// past the row end read 0xFFFF (key 0, below every logit).
//
// issue_chunk starts the 16-byte cp.async copies of the whole vectors (no
// wait); complete_chunk, once they have landed, loads the ragged tail (and
// unaligned rows) with plain loads, pads, applies the penalty patch, and
// returns with the buffer complete.  Both are reached by the whole CTA.
__device__ __forceinline__ void issue_chunk(const KParams& P, uint4* buf, int row, int c, int n) {
  if (!P.vec_ok) return;
  const uint4* s4 = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(P.logits) +
                                                   static_cast<long long>(row) * P.row_stride + c * kSCH);
  const int nfull = n >> 3;
  for (int v = threadIdx.x; v < nfull; v += kThreads) cp_async16(buf + v, s4 + v);
}

template <int DT>
__device__ void complete_chunk(const KParams& P, uint4* buf, int row, int c, int n) {
  using Dt = DType<DT>;
  const int tid = threadIdx.x;
  const int c0 = c * kSCH;
  const uint16_t* src = static_cast<const uint16_t*>(P.logits) + static_cast<long long>(row) * P.row_stride + c0;
  uint16_t* raw = reinterpret_cast<uint16_t*>(buf);
  const int done = P.vec_ok ? ((n >> 3) << 3) : 0;
  for (int i = done + tid; i < kSCH; i += kThreads) raw[i] = (i < n) ? src[i] : static_cast<uint16_t>(0xFFFFu);
  __syncthreads();
  if (P.row_slot) {
    const int slot = P.row_slot[row];
    if (slot >= 0 && slot < P.num_slots) {
      const int len = min(P.slot_len[slot], P.hist_cap);
      const float rf = P.rep_factor ? P.rep_factor[row] : 1.0f;
      const long long base = static_cast<long long>(slot) * P.hist_cap;
      for (int h = tid; h < len; h += kThreads) {
        const int tok = P.hist_tok[base + h];
        const int cnt = P.hist_cnt[base + h];
        const int li = tok - c0;
        if (cnt <= 0 || li < 0 || li >= n) continue;
        const float x = Dt::to_f32(raw[li]);
        const float m = P.hist_mval ? P.hist_mval[base + h] : penalty_divisor<DT>(cnt, rf);
        raw[li] = static_cast<uint16_t>(Dt::to_raw(Dt::round(__fdiv_rn(x, m))));
      }
    }
    __syncthreads();
  }
}

// issue + wait + complete (the finisher's re-reads)
template <int DT>
__device__ void stage_chunk(const KParams& P, uint4* buf, int row, int c, int n) {
  issue_chunk(P, buf, row, c, n);
  cp_async_wait_all();
  __syncthreads();
  complete_chunk<DT>(P, buf, row, c, n);
}

// the 32 keys of this thread, entries 32*tid .. 32*tid+31 of the staged chunk
__device__ __forceinline__ void thread_keys(const uint4* buf, uint32_t (&w)[kSWords]) {
  const uint4* p = buf + threadIdx.x * 4;
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint4 x = p[s];
    w[4 * s + 0] = key16x2(x.x);
    w[4 * s + 1] = key16x2(x.y);
    w[4 * s + 2] = key16x2(x.z);
    w[4 * s + 3] = key16x2(x.w);
  }
}

__device__ __forceinline__ int chunk_len(const KParams& P, int c) { return min(kSCH, P.V - c * kSCH); }

// ------------------------------------------------------- draw in one chunk
// Re-stages chunk c and returns the row index of the first entry (vocab
// order) whose inclusive cumulative mass over keys >= kdraw exceeds rem;
// if rounding leaves rem unreached, the last entry with non-zero mass.
template <int DT>
__device__ __noinline__ int locate_in_chunk(const KParams& P, SSmem& S, uint4* buf, int row, int c, uint32_t kdraw,
                                            float T, float rT, float M, float rem, bool take_last) {
  using C = Codec<DT, 16>;
  const int tid = threadIdx.x;
  const int n = chunk_len(P, c);
  __syncthreads();  // the buffer may still be read by the caller
  stage_chunk<DT>(P, buf, row, c, n);
  uint32_t w[kSWords];
  thread_keys(buf, w);
  const int nv = max(0, min(kSPerT, n - kSPerT * tid));
  float acc = 0.f;
  int lastj = -1;
#pragma unroll
  for (int j = 0; j < kSPerT; ++j) {
    const uint32_t key = ECAH_SKEY(w, j);
    if (j < nv && key >= kdraw) {
      const float e = mass_of(C::value(key), T, rT, M);
      if (e > 0.f) lastj = j;
      acc += e;
    }
  }
  float tot;
  const float excl = sblock_excl_scanf(acc, S.fw, &tot);
  int mine = INT_MAX;
  if (!take_last && acc > 0.f && excl + acc > rem) {
    // the crossing lies in this thread's entries: walk them again in order
    float run = excl;
#pragma unroll
    for (int j = 0; j < kSPerT; ++j) {
      const uint32_t key = ECAH_SKEY(w, j);
      if (mine == INT_MAX && j < nv && key >= kdraw) {
        const float e = mass_of(C::value(key), T, rT, M);
        if (e > 0.f) {
          run += e;
          if (run > rem) mine = kSPerT * tid + j;
        }
      }
    }
    if (mine == INT_MAX) mine = kSPerT * tid + lastj;
  }
  const int pick = sblock_min(mine, S.iw);
  if (pick != INT_MAX) return c * kSCH + pick;
  const int last = sblock_maxi(lastj >= 0 ? kSPerT * tid + lastj : -1, S.iw);
  return c * kSCH + max(last, 0);
}

// Chunk selection for the draw: S.ct[c] holds the kept mass of chunk c.
// Writes S.ib[8] = chosen chunk (-1: no mass), S.ib[9] = take_last,
// S.fb[8] = remaining target inside the chunk, S.fb[9] = Z.
__device__ __forceinline__ void select_chunk(SSmem& S, int NC, float u) {
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < 32) {
    const int ca = 2 * lane, cb = 2 * lane + 1;
    const float a = (ca < NC) ? S.ct[ca] : 0.f;
    const float b = (cb < NC) ? S.ct[cb] : 0.f;
    const float s = a + b;
    float incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    float excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
    if (lane == 0) excl = 0.f;
    const float Z = __shfl_sync(0xFFFFFFFFu, incl, 31);
    const float target = __fmul_rn(u, Z);
    const float cumA = excl + a;
    const bool hitA = a > 0.f && cumA > target;
    const bool hitB = b > 0.f && cumA + b > target;
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, hitA || hitB);
    const unsigned nzm = __ballot_sync(0xFFFFFFFFu, s > 0.f);
    int sel = -1, take_last = 0;
    float before = 0.f;
    if (hit) {
      const int L = __ffs(hit) - 1;
      const bool inA = __shfl_sync(0xFFFFFFFFu, hitA, L);
      const float ex = __shfl_sync(0xFFFFFFFFu, excl, L);
      const float aa = __shfl_sync(0xFFFFFFFFu, a, L);
      sel = inA ? 2 * L : 2 * L + 1;
      before = inA ? ex : ex + aa;
    } else if (nzm) {
      const int L = 31 - __clz(nzm);
      const float bb = __shfl_sync(0xFFFFFFFFu, b, L);
      const float ex = __shfl_sync(0xFFFFFFFFu, excl, L);
      const float aa = __shfl_sync(0xFFFFFFFFu, a, L);
      sel = (bb > 0.f) ? 2 * L + 1 : 2 * L;
      before = (bb > 0.f) ? ex + aa : ex;
      take_last = 1;
    }
    if (lane == 0) {
      S.ib[8] = sel;
      S.ib[9] = take_last;
      S.fb[8] = __fsub_rn(target, before);
      S.fb[9] = Z;
    }
  }
  __syncthreads();
}

// ------------------------------------------------------ candidate staging
// Offsets of the chunk lists when staged back to back (lists are padded to
// whole 16-byte vectors).  Chunks [cb, ce) fill one chunk buffer.
__device__ __forceinline__ void cand_prefix(SSmem& S, int NC) {
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int c = 0; c < NC; ++c) {
      S.pre[c] = acc;
      acc += (S.nc[c] + 3) & ~3;
    }
    S.pre[NC] = acc;
  }
  __syncthreads();
}

__device__ __forceinline__ int cand_batch_end(const SSmem& S, int NC, int cb) {
  int ce = cb + 1;
  while (ce < NC && S.pre[ce + 1] - S.pre[cb] <= kSStage) ++ce;
  return ce;
}

__device__ void stage_cands(const KParams& P, SSmem& S, uint4* buf, int row, int cb, int ce) {
  const int NC = P.NC;
  const int base = S.pre[cb];
  const int nvec = (S.pre[ce] - base) >> 2;
  int cur = cb;
  for (int v = threadIdx.x; v < nvec; v += kThreads) {
    const int e = base + 4 * v;
    while (S.pre[cur + 1] <= e) ++cur;
    const uint4* src = reinterpret_cast<const uint4*>(P.ws_cand + (static_cast<size_t>(row) * NC + cur) * kSCap) +
                       ((e - S.pre[cur]) >> 2);
    cp_async16(buf + v, src);
  }
  cp_async_wait_all();
  __syncthreads();
}

// ---------------------------------------------------- fallback thresholds
// Two-digit radix select (6 | 10 bits) over the whole row, re-read chunk by
// chunk: top-k by counts, top-p by fixed-point level-0 masses then exact
// per-key masses of the selected level-0 bin.  Results in S.ib[12..13].
template <int DT>
__device__ __noinline__ void generic_thresholds(const KParams& P, SSmem& S, uint4* buf, int row, float M, float T, float rT,
                                   uint32_t key_cut, int k_eff, bool topk, float pp, bool topp) {
  using C = Codec<DT, 16>;
  const int NC = P.NC;
  const int tid = threadIdx.x, lane = tid & 31;
  unsigned* h = S.hist;
  uint32_t key_lo_k = 0u;
  if (topk) {
    for (int i = tid; i < kSWin; i += kThreads) h[i] = 0u;
    __syncthreads();
    for (int c = 0; c < NC; ++c) {
      const int n = chunk_len(P, c);
      stage_chunk<DT>(P, buf, row, c, n);
      uint32_t w[kSWords];
      thread_keys(buf, w);
      const int nv = max(0, min(kSPerT, n - kSPerT * tid));
#pragma unroll
      for (int j = 0; j < kSPerT; ++j) {
        const uint32_t key = ECAH_SKEY(w, j);
        if (j < nv) atomicAdd(&h[((key >> 10) << 5) | lane], 1u);
      }
      __syncthreads();
    }
    if (tid < 64) {
      unsigned acc = 0u;
#pragma unroll 8
      for (int j = 0; j < 32; ++j) acc += h[(tid << 5) | ((j + tid) & 31)];
      S.binc[tid] = acc;
    }
    __syncthreads();
    if (tid < 32) {
      int b; unsigned above;
      warp_select_seq<unsigned, 64, true>(S.binc, static_cast<unsigned>(k_eff), &b, &above);
      if (lane == 0) { S.ib[12] = b; S.ib[13] = static_cast<int>(above); }
    }
    __syncthreads();
    const uint32_t b0 = static_cast<uint32_t>(S.ib[12]);
    const unsigned krem = static_cast<unsigned>(k_eff) - static_cast<unsigned>(S.ib[13]);
    for (int i = tid; i < 1024; i += kThreads) h[i] = 0u;
    __syncthreads();
    for (int c = 0; c < NC; ++c) {
      const int n = chunk_len(P, c);
      stage_chunk<DT>(P, buf, row, c, n);
      uint32_t w[kSWords];
      thread_keys(buf, w);
      const int nv = max(0, min(kSPerT, n - kSPerT * tid));
#pragma unroll
      for (int j = 0; j < kSPerT; ++j) {
        const uint32_t key = ECAH_SKEY(w, j);
        if (j < nv && (key >> 10) == b0) atomicAdd(&h[key & 1023u], 1u);
      }
      __syncthreads();
    }
    if (tid < 32) {
      int d; unsigned ab;
      warp_select_seq<unsigned, 1024, true>(h, krem, &d, &ab);
      if (lane == 0) S.ib[12] = static_cast<int>(tie_floor<DT, 16>((b0 << 10) | static_cast<uint32_t>(d), T));
    }
    __syncthreads();
    key_lo_k = static_cast<uint32_t>(S.ib[12]);
    __syncthreads();
  }
  uint32_t key_lo = key_lo_k;
  if (topp) {
    const uint32_t klo = max(key_lo_k, key_cut);
    for (int i = tid; i < kSWin; i += kThreads) h[i] = 0u;
    __syncthreads();
    float sacc = 0.f;
    for (int c = 0; c < NC; ++c) {
      const int n = chunk_len(P, c);
      stage_chunk<DT>(P, buf, row, c, n);
      uint32_t w[kSWords];
      thread_keys(buf, w);
      const int nv = max(0, min(kSPerT, n - kSPerT * tid));
#pragma unroll
      for (int j = 0; j < kSPerT; ++j) {
        const uint32_t key = ECAH_SKEY(w, j);
        if (j < nv && key >= klo) {
          const float e = mass_of(C::value(key), T, rT, M);
          sacc += e;
          atomicAdd(&h[((key >> 10) << 5) | lane], to_fixed(e, kGenFx));
        }
      }
      __syncthreads();
    }
    const float S_K = sblock_sum(sacc, S.fw);
    if (tid < 64) {
      unsigned long long acc = 0ull;
#pragma unroll 8
      for (int j = 0; j < 32; ++j) acc += h[(tid << 5) | ((j + tid) & 31)];
      S.l0f[tid] = static_cast<float>(acc) * kGenFxInv;
    }
    __syncthreads();
    const float target = __fmul_rn(pp, S_K);
    if (tid < 32) {
      int b; float above;
      warp_select_seq<float, 64, true>(S.l0f, target, &b, &above);
      if (lane == 0) S.ib[14] = b;
    }
    __syncthreads();
    const uint32_t b0 = static_cast<uint32_t>(S.ib[14]);
    for (int i = tid; i < 1024; i += kThreads) h[i] = 0u;
    __syncthreads();
    float above = 0.f;  // exact mass of keys in bins above b0
    for (int c = 0; c < NC; ++c) {
      const int n = chunk_len(P, c);
      stage_chunk<DT>(P, buf, row, c, n);
      uint32_t w[kSWords];
      thread_keys(buf, w);
      const int nv = max(0, min(kSPerT, n - kSPerT * tid));
#pragma unroll
      for (int j = 0; j < kSPerT; ++j) {
        const uint32_t key = ECAH_SKEY(w, j);
        if (j < nv && key >= klo) {
          const uint32_t hb = key >> 10;
          if (hb == b0) atomicAdd(&h[key & 1023u], 1u);
          else if (hb > b0) above += mass_of(C::value(key), T, rT, M);
        }
      }
      __syncthreads();
    }
    const float above_b0 = sblock_sum(above, S.fw);
    float* m1 = reinterpret_cast<float*>(buf);
    for (int d = tid; d < 1024; d += kThreads) {
      const uint32_t key = (b0 << 10) | static_cast<uint32_t>(d);
      m1[d] = h[d] ? __fmul_rn(static_cast<float>(h[d]), mass_of(C::value(key), T, rT, M)) : 0.f;
    }
    __syncthreads();
    if (tid < 32) {
      int d; float ab;
      warp_select_seq<float, 1024, true>(m1, __fsub_rn(target, above_b0), &d, &ab);
      if (lane == 0)
        S.ib[13] = static_cast<int>(max(tie_floor<DT, 16>((b0 << 10) | static_cast<uint32_t>(d), T), key_lo_k));
    }
    __syncthreads();
    key_lo = static_cast<uint32_t>(S.ib[13]);
  }
  __syncthreads();
  if (tid == 0) { S.ib[12] = static_cast<int>(key_lo_k); S.ib[13] = static_cast<int>(key_lo); }
  __syncthreads();
}

// ------------------------------------------------------- finishing a row
// Non-greedy rows: thresholds, kept mass, draw.  Returns the sampled index
// (the same on every thread).
template <int DT>
__device__ __noinline__ int finish_sampled(const KParams& P, SSmem& S, uint4* buf, int row, uint32_t kmax, uint32_t F,
                                           float M, float T,
                              int k_eff, bool topk, float pp, bool topp, float u) {
  using C = Codec<DT, 16>;
  const int NC = P.NC;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float rT = __frcp_rn(T);
  const uint32_t key_cut = zero_mass_cut<DT, 16>(M, T);
  const bool cand_mode = topk || topp;
  const int needN = topk ? (k_eff <= kSCap ? k_eff : 0) : (topp ? kSDense : 0);

  // rows without top-k: chunk masses rescaled to the row max
  float S_all = 0.f;
  if (!topk) {
    if (warp == 0) {
      for (int c = lane; c < NC; c += 32) {
        const float sr = S.sr[c];
        S.ps[c] = (sr > 0.f) ? ex2_approx(__fmul_rn(__fsub_rn(S.mr[c], M), kLog2e)) : 0.f;
      }
      __syncwarp();
      if (lane == 0) {
        float a = 0.f;
        for (int c = 0; c < NC; ++c) a += __fmul_rn(S.sr[c], S.ps[c]);
        S.fb[0] = a;
      }
    }
    __syncthreads();
    S_all = S.fb[0];
  }

  bool fast = true;
  uint32_t key_lo_k = 0u, key_lo = 0u;
  bool one_batch = false;
  const unsigned* raw32 = reinterpret_cast<const unsigned*>(buf);
  if (cand_mode) {
    if (needN == 0 || F >= kNoFloor) {
      fast = false;
    } else {
      // exact per-key counts of the candidates with key >= F, bin b = kmax - key
      unsigned* cnt = S.hist;
      for (int i = tid; i < kSWin; i += kThreads) cnt[i] = 0u;
      cand_prefix(S, NC);
      one_batch = S.pre[NC] <= kSStage;
      for (int cb = 0; cb < NC;) {
        const int ce = cand_batch_end(S, NC, cb);
        stage_cands(P, S, buf, row, cb, ce);
        const int ne = S.pre[ce] - S.pre[cb];
        for (int i = tid; i < ne; i += kThreads) {
          const unsigned x = raw32[i];
          const uint32_t key = x >> 16;
          if ((x & 0xFFFFu) != kSentinel && key >= F) atomicAdd(&cnt[kmax - key], 1u);
        }
        __syncthreads();
        cb = ce;
      }
      const int Bmax = static_cast<int>(kmax - F);
      if (topk) {
        if (tid < 32) {
          unsigned tot = 0u;
          for (int b = lane; b < kSWin; b += 32) tot += cnt[b];
          tot = __reduce_add_sync(0xFFFFFFFFu, tot);
          int b; unsigned above;
          warp_select_seq<unsigned, kSWin, false>(cnt, static_cast<unsigned>(k_eff), &b, &above);
          if (lane == 0) {
            int ok = tot >= static_cast<unsigned>(k_eff);
            uint32_t klk = 0u;
            if (ok) {
              klk = tie_floor<DT, 16>(kmax - static_cast<uint32_t>(b), T);
              ok = klk >= F;
            }
            S.ib[2] = ok;
            S.ib[3] = static_cast<int>(klk);
          }
        }
        __syncthreads();
        fast = S.ib[2] != 0;
        key_lo_k = static_cast<uint32_t>(S.ib[3]);
      }
      key_lo = key_lo_k;
      if (fast && topp) {
        // bin masses (count * mass of one entry), in place over the counts
        const int bk = topk ? static_cast<int>(kmax - key_lo_k) : Bmax;
        float* mb = reinterpret_cast<float*>(S.hist);
        for (int b = tid; b < kSWin; b += kThreads) {
          const unsigned cn = cnt[b];
          float m = 0.f;
          if (b <= bk && cn) m = __fmul_rn(static_cast<float>(cn), mass_of(C::value(kmax - static_cast<uint32_t>(b)), T, rT, M));
          mb[b] = m;
        }
        __syncthreads();
        if (tid < 32) {
          float s = 0.f;
          for (int b = lane; b < kSWin; b += 32) s += mb[b];
          s = warp_sum(s);
          const float S_K = topk ? s : S_all;
          const float target = __fmul_rn(pp, S_K);
          int b; float above;
          warp_select_seq<float, kSWin, false>(mb, target, &b, &above);
          if (lane == 0) {
            int ok = s >= target;
            uint32_t kl = 0u;
            if (ok) {
              kl = max(tie_floor<DT, 16>(kmax - static_cast<uint32_t>(b), T), key_lo_k);
              ok = kl >= F;
            }
            S.ib[2] = ok;
            S.ib[3] = static_cast<int>(kl);
          }
        }
        __syncthreads();
        fast = S.ib[2] != 0;
        key_lo = static_cast<uint32_t>(S.ib[3]);
      }
      __syncthreads();
    }
  }

  if (!fast) {
    generic_thresholds<DT>(P, S, buf, row, M, T, rT, key_cut, k_eff, topk, pp, topp);
    key_lo_k = static_cast<uint32_t>(S.ib[12]);
    key_lo = static_cast<uint32_t>(S.ib[13]);
  }
  const uint32_t kdraw = max(key_lo, key_cut);

  // kept mass per chunk
  if (fast && cand_mode) {
    for (int cb = 0; cb < NC;) {
      const int ce = cand_batch_end(S, NC, cb);
      if (!one_batch) stage_cands(P, S, buf, row, cb, ce);
      for (int c = cb + warp; c < ce; c += kWarps) {
        const unsigned* L = raw32 + (S.pre[c] - S.pre[cb]);
        const int nc = S.nc[c];
        float a = 0.f;
        for (int i = lane; i < nc; i += 32) {
          const uint32_t key = L[i] >> 16;
          if (key >= kdraw) a += mass_of(C::value(key), T, rT, M);
        }
        a = warp_sum(a);
        if (lane == 0) S.ct[c] = a;
      }
      __syncthreads();
      cb = ce;
    }
  } else if (fast) {
    for (int c = tid; c < NC; c += kThreads) S.ct[c] = __fmul_rn(S.sr[c], S.ps[c]);
    __syncthreads();
  } else {
    for (int c = 0; c < NC; ++c) {
      const int n = chunk_len(P, c);
      stage_chunk<DT>(P, buf, row, c, n);
      uint32_t w[kSWords];
      thread_keys(buf, w);
      const int nv = max(0, min(kSPerT, n - kSPerT * tid));
      float a = 0.f;
#pragma unroll
      for (int j = 0; j < kSPerT; ++j) {
        const uint32_t key = ECAH_SKEY(w, j);
        if (j < nv && key >= kdraw) a += mass_of(C::value(key), T, rT, M);
      }
      a = sblock_sum(a, S.fw);
      if (tid == 0) S.ct[c] = a;
    }
    __syncthreads();
  }

  select_chunk(S, NC, u);
  const int csel = S.ib[8];
  const bool take_last = S.ib[9] != 0;
  float rem = S.fb[8];
  const float Z = S.fb[9];
  int result;
  if (csel < 0) {
    // no finite mass anywhere: the lowest index of the row max
    if (warp == 0) {
      int f = INT_MAX;
      for (int c = lane; c < NC; c += 32)
        if (S.lm[c] == kmax) f = min(f, S.fi[c]);
      f = __reduce_min_sync(0xFFFFFFFFu, f);
      if (lane == 0) S.ib[10] = (f == INT_MAX) ? 0 : f;
    }
    __syncthreads();
    result = S.ib[10];
  } else if (fast && cand_mode) {
    // inverse CDF over the chosen chunk's candidates, in vocab order
    const int nc = S.nc[csel];
    const unsigned* L;
    if (one_batch) {
      L = raw32 + S.pre[csel];
    } else {
      __syncthreads();
      stage_cands(P, S, buf, row, csel, csel + 1);
      L = raw32;
    }
    int pick = INT_MAX, last = -1;
    for (int base = 0; base < nc && pick == INT_MAX; base += kThreads) {
      const int i = base + tid;
      float e = 0.f;
      if (i < nc) {
        const uint32_t key = L[i] >> 16;
        if (key >= kdraw) e = mass_of(C::value(key), T, rT, M);
      }
      float tot;
      const float excl = sblock_excl_scanf(e, S.fw, &tot);
      const int mine = (!take_last && e > 0.f && excl + e > rem) ? i : INT_MAX;
      pick = sblock_min(mine, S.iw);
      last = max(last, sblock_maxi(e > 0.f ? i : -1, S.iw));
      rem = __fsub_rn(rem, tot);
    }
    const int at = (pick != INT_MAX) ? pick : max(last, 0);
    result = csel * kSCH + static_cast<int>(L[at] & 0xFFFFu);
  } else {
    result = locate_in_chunk<DT>(P, S, buf, row, csel, kdraw, T, rT, M, rem, take_last);
  }

  if (tid == 0) {
    if (P.row_stats) {
      float* st = P.row_stats + 4ll * row;
      st[0] = topk ? C::value(key_lo_k) : -INFINITY;
      st[1] = (topk || topp) ? C::value(key_lo) : -INFINITY;
      st[2] = M;
      st[3] = Z;
    }
    RowFin* fin = static_cast<RowFin*>(P.ws_fin) + row;
    fin->M = M;
    fin->Z = Z;
    fin->kdraw = kdraw;
    fin->mode = (csel < 0) ? 2 : 0;
    fin->idx = result;
  }
  return result;
}

template <int DT>
__device__ __noinline__ void finish_row(const KParams& P, SSmem& S, uint4* buf, int row) {
  using C = Codec<DT, 16>;
  const int NC = P.NC;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ChunkSum* cs = static_cast<const ChunkSum*>(P.ws_sums) + static_cast<size_t>(row) * NC;
  const float T = P.temperature[row];
  const int kk = P.top_k[row];
  const int k_eff = (kk <= 0 || kk >= P.V) ? P.V : kk;
  const float pp = P.top_p[row];
  const bool topk = k_eff < P.V;
  const bool topp = (pp > 0.f && pp < 1.f);
  float u;
  if (P.uniforms) u = P.uniforms[row];
  else u = row_uniform(__ldcg(&P.philox_state[0]), __ldcg(&P.philox_state[1]), static_cast<uint64_t>(row));

  if (warp == 0) {
    unsigned km = 0u, fl = 0u;
    for (int c = lane; c < NC; c += 32) {
      const unsigned lm = __ldcg(&cs[c].lmax);
      const unsigned f = __ldcg(&cs[c].floor);
      S.lm[c] = lm;
      S.nc[c] = __ldcg(&cs[c].ncand);
      S.fi[c] = __ldcg(&cs[c].first);
      S.mr[c] = __ldcg(&cs[c].mref);
      S.sr[c] = __ldcg(&cs[c].sref);
      km = max(km, lm);
      fl = max(fl, f);
    }
    km = __reduce_max_sync(0xFFFFFFFFu, km);
    fl = __reduce_max_sync(0xFFFFFFFFu, fl);
    if (lane == 0) { S.ib[0] = static_cast<int>(km); S.ib[1] = static_cast<int>(fl); }
  }
  __syncthreads();
  const uint32_t kmax = static_cast<uint32_t>(S.ib[0]);
  const uint32_t F = static_cast<uint32_t>(S.ib[1]);
  const float ymax = C::value(kmax);
  const float M = __fdiv_rn(ymax, T);
  const bool greedy = !(T > 0.f) || !isfinite(M);
  int result;
  if (greedy) {
    if (warp == 0) {
      int f = INT_MAX;
      for (int c = lane; c < NC; c += 32)
        if (S.lm[c] == kmax) f = min(f, S.fi[c]);
      f = __reduce_min_sync(0xFFFFFFFFu, f);
      if (lane == 0) S.ib[2] = (f == INT_MAX) ? 0 : f;
    }
    __syncthreads();
    result = S.ib[2];
    if (tid == 0) {
      if (P.row_stats) {
        float* st = P.row_stats + 4ll * row;
        st[0] = ymax; st[1] = ymax; st[2] = ymax; st[3] = 1.0f;
      }
      RowFin* fin = static_cast<RowFin*>(P.ws_fin) + row;
      fin->M = ymax;
      fin->Z = 1.0f;
      fin->kdraw = 0u;
      fin->mode = 1;
      fin->idx = result;
    }
  } else {
    result = finish_sampled<DT>(P, S, buf, row, kmax, F, M, T, k_eff, topk, pp, topp, u);
  }
  if (tid == 0) {
    P.out[row] = min(result, P.V - 1);
    if (!P.uniforms) {
      // the last row to finish advances the Philox offset; every row read
      // the offset before it arrives here
      __threadfence();
      const unsigned prev = atomicAdd(P.done_counter, 1u);
      if (prev == static_cast<unsigned>(P.B) - 1u) {
        P.philox_state[1] += 1ull;
        *P.done_counter = 0u;
        __threadfence();
      }
    }
  }
}

// ------------------------------------------------------------ the kernel
// One staged chunk of one row: keys, chunk max, candidates or chunk mass,
// summary, arrival; the chunk that arrives last at its row finishes the row.
template <int DT>
__device__ __forceinline__ void process_chunk(const KParams& P, SSmem& S, uint4* buf, int row, int c, int n) {
  using C = Codec<DT, 16>;
  const int NC = P.NC;
  const int tid = threadIdx.x, lane = tid & 31;
  const int c0 = c * kSCH;
  const float T = P.temperature[row];
  const int kk = P.top_k[row];
  const int k_eff = (kk <= 0 || kk >= P.V) ? P.V : kk;
  const float pp = P.top_p[row];
  const bool topk = k_eff < P.V;
  const bool topp = (pp > 0.f && pp < 1.f);
  const bool sampled = T > 0.f;

  uint32_t w[kSWords];
  thread_keys(buf, w);
  const int nv = max(0, min(kSPerT, n - kSPerT * tid));
  uint32_t tm = 0u;
#pragma unroll
  for (int j = 0; j < kSWords; ++j) tm = __vmaxu2(tm, w[j]);
  tm = max(tm & 0xFFFFu, tm >> 16);
  const uint32_t lmax = sblock_max(tm, S.uw);  // padding keys are 0: never above a logit

  int first = INT_MAX;
  if (tm == lmax) {
#pragma unroll
    for (int j = 0; j < kSPerT; ++j)
      if (first == INT_MAX && j < nv && ECAH_SKEY(w, j) == lmax) first = kSPerT * tid + j;
  }
  first = sblock_min(first, S.iw);

  const int needN = !sampled ? 0 : (topk ? (k_eff <= kSCap ? k_eff : 0) : (topp ? kSDense : 0));
  unsigned floor = kNoFloor;
  int ncand = 0;
  if (needN > 0) {
    for (int i = tid; i < kSWin; i += kThreads) S.hist[i] = 0u;
    __syncthreads();
    // counts of the 2048 keys below the chunk max, in bins of 32 keys
    const uint32_t lo = (lmax >= static_cast<uint32_t>(kSWin - 1)) ? lmax - static_cast<uint32_t>(kSWin - 1) : 0u;
#pragma unroll
    for (int j = 0; j < kSPerT; ++j) {
      const uint32_t key = ECAH_SKEY(w, j);
      if (j < nv && key >= lo) atomicAdd(&S.hist[(((lmax - key) >> 5) << 5) | static_cast<uint32_t>(lane)], 1u);
    }
    __syncthreads();
    if (tid < kSBins) {
      unsigned acc = 0u;
#pragma unroll 8
      for (int j = 0; j < 32; ++j) acc += S.hist[(tid << 5) | ((j + tid) & 31)];
      S.binc[tid] = acc;
    }
    __syncthreads();
    if (tid < 32) {
      const unsigned a = S.binc[2 * lane], b = S.binc[2 * lane + 1];
      unsigned incl = a + b;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      const unsigned cumA = incl - b, cumB = incl;  // counts of bins 0..2l and 0..2l+1
      const unsigned N = static_cast<unsigned>(needN);
      const unsigned hit = __ballot_sync(0xFFFFFFFFu, cumB >= N);
      int bstar = kSBins - 1;
      if (hit) {
        const int L = __ffs(hit) - 1;
        bstar = (__shfl_sync(0xFFFFFFFFu, cumA, L) >= N) ? 2 * L : 2 * L + 1;
      }
      unsigned cst = (bstar & 1) ? __shfl_sync(0xFFFFFFFFu, cumB, bstar >> 1) : __shfl_sync(0xFFFFFFFFu, cumA, bstar >> 1);
      if (cst > static_cast<unsigned>(kSCap)) {
        // the counts grow with the bin: keep the longest prefix of bins that fits
        const int nfit = __popc(__ballot_sync(0xFFFFFFFFu, cumA <= static_cast<unsigned>(kSCap))) +
                         __popc(__ballot_sync(0xFFFFFFFFu, cumB <= static_cast<unsigned>(kSCap)));
        bstar = nfit - 1;
        const int sl = bstar >= 0 ? (bstar >> 1) : 0;
        const unsigned va = __shfl_sync(0xFFFFFFFFu, cumA, sl), vb = __shfl_sync(0xFFFFFFFFu, cumB, sl);
        cst = bstar >= 0 ? ((bstar & 1) ? vb : va) : 0u;
      }
      if (lane == 0) {
        unsigned fl = kNoFloor;
        if (bstar >= 0) {
          const unsigned d = static_cast<unsigned>(bstar) * 32u + 31u;
          fl = (d <= lmax) ? max(lmax - d, lo) : lo;
        }
        S.ib[0] = static_cast<int>(fl);
        S.ib[1] = static_cast<int>(cst);
      }
    }
    __syncthreads();
    floor = static_cast<unsigned>(S.ib[0]);
    ncand = S.ib[1];
    if (floor != kNoFloor) {
      // the entries with key >= floor, written in vocab order
      int cnt = 0;
#pragma unroll
      for (int j = 0; j < kSPerT; ++j) cnt += (j < nv && ECAH_SKEY(w, j) >= floor) ? 1 : 0;
      int total;
      const int off = sblock_excl_scan(cnt, S.iw, &total);
      unsigned* list = P.ws_cand + (static_cast<size_t>(row) * NC + c) * kSCap;
      unsigned* dst = list + off;
      int o = 0;
#pragma unroll
      for (int j = 0; j < kSPerT; ++j) {
        const uint32_t key = ECAH_SKEY(w, j);
        if (j < nv && key >= floor) {
          dst[o] = (key << 16) | static_cast<uint32_t>(kSPerT * tid + j);
          ++o;
        }
      }
      if (tid == 0)
        for (int i = total; i < ((total + 3) & ~3); ++i) list[i] = kSentinel;
    }
  }

  float mref = 0.f, sref = 0.f;
  if (sampled && !topk) {
    // softmax mass of the chunk relative to its own max
    mref = __fdiv_rn(C::value(lmax), T);
    if (isfinite(mref)) {
      const uint32_t cut = zero_mass_cut<DT, 16>(mref, T);
      const float rT = __frcp_rn(T);
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < kSPerT; ++j) {
        const uint32_t key = ECAH_SKEY(w, j);
        if (j < nv && key >= cut) acc += mass_of(C::value(key), T, rT, mref);
      }
      sref = sblock_sum(acc, S.fw);
    }
  }

  if (tid == 0) {
    ChunkSum* cs = static_cast<ChunkSum*>(P.ws_sums) + static_cast<size_t>(row) * NC + c;
    cs->lmax = lmax;
    cs->floor = floor;
    cs->ncand = ncand;
    cs->first = (first == INT_MAX) ? INT_MAX : c0 + first;
    cs->mref = mref;
    cs->sref = sref;
  }
}

// Persistent: CTA b takes units b, b + G, b + 2G, ... (unit = row * NC + chunk)
// and copies unit i+1 into the other buffer while it works on unit i.
template <int DT>
__global__ void __launch_bounds__(kThreads, 4) stream_scan_kernel(const __grid_constant__ KParams P) {
  __shared__ SSmem S;
  const int NC = P.NC;
  const int units = P.B * NC;
  const int G = static_cast<int>(gridDim.x);
  int u = static_cast<int>(blockIdx.x);
  if (u >= units) return;
  issue_chunk(P, S.raw[0], u / NC, u % NC, chunk_len(P, u % NC));
  cp_async_commit();
  for (int i = 0; u < units; ++i, u += G) {
    const int un = u + G;
    uint4* cur = S.raw[i & 1];
    if (un < units) {
      issue_chunk(P, S.raw[(i + 1) & 1], un / NC, un % NC, chunk_len(P, un % NC));
      cp_async_commit();
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    __syncthreads();
    const int row = u / NC;
    const int c = u - row * NC;
    const int n = chunk_len(P, c);
    complete_chunk<DT>(P, cur, row, c, n);
    process_chunk<DT>(P, S, cur, row, c, n);
    __syncthreads();  // `cur` is refilled two units on
  }
}

// One CTA per row, launched after stream_scan_kernel: merges the row's chunk
// summaries and draws.
template <int DT>
__global__ void __launch_bounds__(kThreads, 1) stream_finish_kernel(const __grid_constant__ KParams P) {
  __shared__ SSmem S;
  finish_row<DT>(P, S, S.raw[0], static_cast<int>(blockIdx.x));
}

// probs_out of the rows finished by stream_finish_kernel (launched after it)
template <int DT>
__global__ void __launch_bounds__(kThreads) stream_probs_kernel(const __grid_constant__ KParams P) {
  using C = Codec<DT, 16>;
  __shared__ uint4 buf[kSVecs];
  const int NC = P.NC;
  const int row = blockIdx.x / NC;
  const int c = blockIdx.x - row * NC;
  const int c0 = c * kSCH;
  const int n = chunk_len(P, c);
  const RowFin f = static_cast<const RowFin*>(P.ws_fin)[row];
  float* po = P.probs_out + static_cast<long long>(row) * P.V + c0;
  if (f.mode != 0) {
    for (int i = threadIdx.x; i < n; i += kThreads) po[i] = (f.mode == 1 && c0 + i == f.idx) ? 1.0f : 0.0f;
    return;
  }
  stage_chunk<DT>(P, buf, row, c, n);
  const float T = P.temperature[row];
  const float rT = __frcp_rn(T);
  const uint16_t* raw = reinterpret_cast<const uint16_t*>(buf);
  for (int i = threadIdx.x; i < n; i += kThreads) {
    const uint32_t key = key16(raw[i]);
    po[i] = (key >= f.kdraw) ? __fdiv_rn(mass_of(C::value(key), T, rT, f.M), f.Z) : 0.0f;
  }
}

#undef ECAH_SKEY

}  // namespace ecah
