// Row-per-CTA token sampler for sm_100a: one 1024-thread CTA owns a row (or,
// for batches that leave SMs idle, a run of the row's rounds, see
// part_exchange), streams it from HBM through one four-stage cp.async
// pipeline per warp (32 KB rounds, a 1 KB slice per warp), keeps every
// running quantity on chip and finishes the row without waiting on any other
// CTA.
//
// During the stream, per row mode (16-bit keys: fp16/bf16 logits):
//   - every row: per-thread running (max key, first round holding it);
//   - unsplit rows with top-k: per chunk of 16 entries its top key (records;
//     lean_finish); unsplit rows with top-p and no top-k: per chunk its two
//     top keys, counted into a per-key histogram as they stream
//     (plean_finish); either finishes without re-streaming the row;
//   - other rows with top-k (k <= kMaxN) or top-p: a candidate buffer in shared
//     memory holding, in vocab order, every entry whose key is >= a running
//     floor f.  f starts at the N0-th largest key of the first round (N0 = k
//     for top-k rows; for top-p-only rows kDenseN scaled to the round's share
//     of the row) and is raised, when the buffer would overflow, to the N-th
//     largest key of the buffer and the round's survivors; the buffer always
//     holds exactly the entries seen so far with key >= f, so every entry of
//     the row at or above the final f is a candidate;
//   - rows without top-k: softmax masses per (round, warp) segment, each
//     relative to the segment's own max z, so no mass overflows at any
//     temperature; warps whose keys all lie 36 T below the first round's max
//     skip them (their total mass is below 1e-9 of S).
// After the stream the row max M, the thresholds (exact per-key counts of the
// candidates, as in the cluster kernel's window path) and the draw (inverse
// CDF over the candidates in vocab order, or over segment sums and then one
// re-loaded 512-entry segment) need no further HBM traffic.  Rows whose
// thresholds fall below the candidate floor re-stream the row and run a
// two-digit (8 | 8 bit) radix select.
//
// Op order, masses (mass_of), tie floors and zero-mass cut are those of the
// cluster kernel (sampler_kernel.cuh).
#pragma once

#include <cstddef>
#include <type_traits>

#include "stream_kernel.cuh"

namespace ecah {
namespace rk {

constexpr int kT = 1024;                  // threads per CTA
constexpr int kNW = kT / 32;              // warps
constexpr int kEPT = 16;                  // entries per thread per round
constexpr int kRound = kT * kEPT;         // entries per round (32 KB of fp16)
constexpr int kRVecs = kRound / 8;        // 16-byte vectors per round
constexpr int kStages = 4;                // rounds in flight while one is processed: 3
constexpr int kCB = 8192;                 // candidate buffer entries
constexpr int kMaxN = kCB / 2;            // largest candidate target
constexpr int kDenseN = 4096;             // candidate target of top-p-only rows
constexpr int kHB = 4096;                 // finishing histogram: keys below the row max
constexpr int kMaxRounds = 32;            // vocab <= 32 * 16384
constexpr int kSegs = kMaxRounds * kNW;   // (round, warp) segments of 512 entries
constexpr int kPenCap = 896;              // history entries bucketed in shared memory per row
// fallback level-0 fixed point: a mass <= 1 times 2^22 stays below the 2^23
// to_fixed needs, and a lane's slot sums at most 16 * 32 masses (< 2^32)
constexpr float kFx = 4194304.0f;
constexpr float kFxInv = 1.0f / 4194304.0f;

struct RSmem {
  uint4 stage[kStages][kRVecs];   // pipeline; after the stream: finishing histograms
  unsigned lp[256 * 32];          // lane-private 256-bin histograms
  uint16_t ckey[kCB];             // candidates: key
  uint32_t cidx[kCB];             //             row index
  float ss[kSegs];                // segment masses relative to the segment's reference
  float sq[kSegs];                //   and that reference (z of the segment's max, times log2 e)
  unsigned h256[256];
  unsigned red[2][kNW];           // reduction scratch, alternating
  int wcnt[2][kNW];
  int ib[16];
  float fb[16];
  float part[kNW];                // per-warp partial sums carried across a barrier
  unsigned pend[kMaxRounds];      // split rows: end of each part's candidates in the merged order
  // the row's repetition-penalty history bucketed by slice (round, warp):
  // slice s holds entries [poff[s], poff[s + 1]) of pent
  uint16_t poff[kMaxRounds * kNW + 1];
  uint2 pent[kPenCap];            // {offset in the slice | raw m << 16, additive term a as float bits}
  unsigned long long pre[2];      // the Philox state and
  float upre;                     //   the caller's uniform, copied in while the row streams
  int pen_ok;                     // the buckets hold the whole history
};

// ------------------------------------------------------------ reductions
// Every thread of the CTA calls them in the same order; `ph` alternates the
// scratch so no trailing barrier is needed.
__device__ __forceinline__ unsigned rmax_u(unsigned v, RSmem& S, int& ph) {
  v = __reduce_max_sync(0xFFFFFFFFu, v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) S.red[ph][warp] = v;
  __syncthreads();
  unsigned m = __reduce_max_sync(0xFFFFFFFFu, S.red[ph][lane]);
  ph ^= 1;
  return m;
}

__device__ __forceinline__ unsigned rmin_u(unsigned v, RSmem& S, int& ph) {
  v = __reduce_min_sync(0xFFFFFFFFu, v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) S.red[ph][warp] = v;
  __syncthreads();
  unsigned m = __reduce_min_sync(0xFFFFFFFFu, S.red[ph][lane]);
  ph ^= 1;
  return m;
}

// block max of a and of b behind one barrier
__device__ __forceinline__ void rmax2_u(unsigned a, unsigned b, RSmem& S, int& ph, unsigned* ma, unsigned* mb) {
  a = __reduce_max_sync(0xFFFFFFFFu, a);
  b = __reduce_max_sync(0xFFFFFFFFu, b);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { S.red[ph][warp] = a; S.wcnt[ph][warp] = static_cast<int>(b); }
  __syncthreads();
  *ma = __reduce_max_sync(0xFFFFFFFFu, S.red[ph][lane]);
  *mb = __reduce_max_sync(0xFFFFFFFFu, static_cast<unsigned>(S.wcnt[ph][lane]));
  ph ^= 1;
}

// block min of a and block max of b behind one barrier
__device__ __forceinline__ void rminmax_u(unsigned a, unsigned b, RSmem& S, int& ph, unsigned* mn, unsigned* mx) {
  a = __reduce_min_sync(0xFFFFFFFFu, a);
  b = __reduce_max_sync(0xFFFFFFFFu, b);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { S.red[ph][warp] = a; S.wcnt[ph][warp] = static_cast<int>(b); }
  __syncthreads();
  *mn = __reduce_min_sync(0xFFFFFFFFu, S.red[ph][lane]);
  *mx = __reduce_max_sync(0xFFFFFFFFu, static_cast<unsigned>(S.wcnt[ph][lane]));
  ph ^= 1;
}

// sum in warp order, then lane order (deterministic)
__device__ __forceinline__ float rsum_f(float v, RSmem& S, int& ph) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) S.red[ph][warp] = __float_as_uint(v);
  __syncthreads();
  float t = warp_sum(__uint_as_float(S.red[ph][lane]));
  ph ^= 1;
  return t;
}

// exclusive prefix of v over threads in thread order; *total = sum.  Warps
// whose v are all 0 skip the lane scan; the prefix over warps and the total
// are two warp reductions of the per-warp sums.
__device__ __forceinline__ int rscan_i(int v, RSmem& S, int& ph, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
  if (__any_sync(0xFFFFFFFFu, v != 0)) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
  }
  if (lane == 31) S.wcnt[ph][warp] = incl;
  __syncthreads();
  const int wv = S.wcnt[ph][lane];
  const int base = static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(lane < warp ? wv : 0)));
  *total = static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(wv)));
  ph ^= 1;
  return base + incl - v;
}

__device__ __forceinline__ float rscan_f(float v, RSmem& S, int& ph, float* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) S.red[ph][warp] = __float_as_uint(incl);
  __syncthreads();
  const float wv = __uint_as_float(S.red[ph][lane]);
  float winc = wv;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xFFFFFFFFu, winc, o);
    if (lane >= o) winc += y;
  }
  const float base = __shfl_sync(0xFFFFFFFFu, winc - wv, warp);
  *total = __shfl_sync(0xFFFFFFFFu, winc, 31);
  ph ^= 1;
  return base + (incl - v);
}

// key j (0..15) of a thread's 8 packed key words
#define ECAH_RKEY(w, j) ((((j) & 1) != 0) ? ((w)[(j) >> 1] >> 16) : ((w)[(j) >> 1] & 0xFFFFu))

// ------------------------------------------------------------ the stream
// Round r of `row`: entries [r * kRound, ...) of the row, n of them valid.
__device__ __forceinline__ int round_len(int V, int r) { return min(kRound, V - r * kRound); }

// Per-warp streaming: warp w owns entries [r * kRound + 512 w, + 512) of
// every round r (lane l: 16 l .. 16 l + 15 of them) and four private 1 KB
// stages; it waits only for its own copies, so warps never wait on one
// another while the row streams.
constexpr int kWS = kRound / kNW;         // entries of a warp slice (512)
constexpr int kWV = kWS / 8;              // 16-byte chunks of a slice (64)


// first row entry of this warp's slice of round r, and how many lie in the row
__device__ __forceinline__ int slice_e0(int r) { return r * kRound + (threadIdx.x >> 5) * kWS; }
__device__ __forceinline__ int slice_len(int V, int r) { return max(0, min(kWS, V - slice_e0(r))); }

// Whether the row has a repetition-penalty history to patch in.
__device__ __forceinline__ bool row_has_penalty(const KParams& P, int row) {
  if (!P.row_slot) return false;
  const int slot = P.row_slot[row];
  return slot >= 0 && slot < P.num_slots && min(P.slot_len[slot], P.hist_cap) > 0;
}

// Ragged tail / unaligned rows with plain loads, padding (key 0), penalty
// patch, for this warp's slice.  Returns with the slice complete for the warp.
template <int DT>
__device__ void complete_slice(const KParams& P, const RSmem& S, uint4* st, int row, int r, bool pen) {
  using Dt = DType<DT>;
  const int lane = threadIdx.x & 31;
  const int n = slice_len(P.V, r);
  const int e0 = slice_e0(r);
  const uint16_t* src = static_cast<const uint16_t*>(P.logits) + logits_row_offset(P, row) + e0;
  uint16_t* raw = reinterpret_cast<uint16_t*>(st);
  const int done = P.vec_ok ? ((n >> 3) << 3) : 0;
  if (done < kWS) {
    for (int i = done + lane; i < kWS; i += 32) raw[i] = (i < n) ? src[i] : static_cast<uint16_t>(0xFFFFu);
    __syncwarp();
  }
  if (pen) {
    if (S.pen_ok) {
      // this slice's bucket of the history (shared memory)
      const int sl = r * kNW + (threadIdx.x >> 5);
      for (int i = S.poff[sl] + lane; i < S.poff[sl + 1]; i += 32) {
        const uint2 e = S.pent[i];
        const unsigned o = e.x & 0xFFFFu;
        raw[o] = static_cast<uint16_t>(Dt::to_raw(penalise<DT>(Dt::to_f32(raw[o]), Dt::to_f32(e.x >> 16), __uint_as_float(e.y))));
      }
    } else {
      const int slot = P.row_slot[row];
      const int len = min(P.slot_len[slot], P.hist_cap);
      const float rf = P.rep_factor ? P.rep_factor[row] : 1.0f;
      const long long base = static_cast<long long>(slot) * P.hist_cap;
      for (int h = lane; h < len; h += 32) {
        const int li = P.hist_tok[base + h] - P.vocab_offset - e0;
        const int cnt = P.hist_cnt[base + h];
        if (cnt <= 0 || li < 0 || li >= n) continue;
        const float x = Dt::to_f32(raw[li]);
        const float m = P.hist_mval ? P.hist_mval[base + h] : penalty_divisor<DT>(cnt, rf);
        raw[li] = static_cast<uint16_t>(Dt::to_raw(penalise<DT>(x, m, additive_term(P, row, cnt))));
      }
    }
    __syncwarp();
  }
}

// Buckets the row's penalty history by slice in shared memory (counting sort
// by token / 512), so each warp patches only its slice's entries every round.
// Every thread calls it; S.pen_ok = 0 when the history does not fit (the
// patch then scans the history in global memory).
template <int DT>
__device__ void bucket_penalties(const KParams& P, RSmem& S, int row, int& ph) {
  const int tid = threadIdx.x;
  const int slot = P.row_slot[row];
  const int len = min(P.slot_len[slot], P.hist_cap);
  const float rf = P.rep_factor ? P.rep_factor[row] : 1.0f;
  const long long base = static_cast<long long>(slot) * P.hist_cap;
  const int nsl = (P.V + kWS - 1) / kWS;   // slices of the row
  unsigned* cnt = S.lp;                    // scratch counters, one per slice
  for (int i = tid; i < nsl; i += kT) cnt[i] = 0u;
  __syncthreads();
  for (int h = tid; h < len; h += kT) {
    const int tok = P.hist_tok[base + h] - P.vocab_offset;
    if (P.hist_cnt[base + h] > 0 && tok >= 0 && tok < P.V) atomicAdd(&cnt[tok / kWS], 1u);
  }
  __syncthreads();
  int total;
  const int v = tid < nsl ? static_cast<int>(cnt[tid]) : 0;   // nsl <= kT
  const int off = rscan_i(v, S, ph, &total);
  // slices past the row end (padding of the last round) get empty buckets
  for (int i = tid; i <= kMaxRounds * kNW; i += kT) S.poff[i] = static_cast<uint16_t>(min(i < nsl ? off : total, kPenCap));
  if (tid < nsl) cnt[tid] = static_cast<unsigned>(off);
  if (tid == 0) S.pen_ok = total <= kPenCap;
  __syncthreads();
  if (total <= kPenCap) {
    for (int h = tid; h < len; h += kT) {
      const int tok = P.hist_tok[base + h] - P.vocab_offset;
      const int c = P.hist_cnt[base + h];
      if (c > 0 && tok >= 0 && tok < P.V) {
        const float m = P.hist_mval ? P.hist_mval[base + h] : penalty_divisor<DT>(c, rf);
        // m is a model-dtype value: its 16-bit raw word rides beside the offset
        S.pent[atomicAdd(&cnt[tok / kWS], 1u)] =
            make_uint2(static_cast<unsigned>(tok % kWS) | (DType<DT>::to_raw(m) << 16),
                       __float_as_uint(additive_term(P, row, c)));
      }
    }
  }
  __syncthreads();
}

// Two 16-bit raws -> two order-preserving keys (key16 on each half): prmt
// replicates each half's sign bit over the half, one lop3 applies it.
__device__ __forceinline__ uint32_t keys2(uint32_t w) {
  uint32_t m;
  asm("prmt.b32 %0, %1, 0, 0xBB99;" : "=r"(m) : "r"(w));
  return w ^ (m | 0x80008000u);
}

__device__ __forceinline__ uint32_t max16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t min16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// per half of a key word: 1 where key >= f, else 0 (fm2 = (f - 1) in both
// halves, f >= 1): max(key, f - 1) - (f - 1) is positive exactly there, and
// no half borrows from the other
__device__ __forceinline__ uint32_t surv2(uint32_t w, uint32_t fm2) {
  return min16x2(max16x2(w, fm2) - fm2, 0x00010001u);
}

// the two logits of a raw word as float32 (exact)
template <int DT> __device__ __forceinline__ float2 vals2(uint32_t w);
template <> __device__ __forceinline__ float2 vals2<ECAH_DTYPE_F16>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <> __device__ __forceinline__ float2 vals2<ECAH_DTYPE_BF16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// this thread's 16 raw logits (entries 16 lane .. 16 lane + 15 of its warp's
// slice) and keys
__device__ __forceinline__ void round_load(const uint4* st, uint32_t (&raw)[8], uint32_t (&w)[8]) {
  const int lane = threadIdx.x & 31;
  const uint4 a = st[2 * lane], b = st[2 * lane + 1];
  raw[0] = a.x; raw[1] = a.y; raw[2] = a.z; raw[3] = a.w;
  raw[4] = b.x; raw[5] = b.y; raw[6] = b.z; raw[7] = b.w;
#pragma unroll
  for (int j = 0; j < 8; ++j) w[j] = keys2(raw[j]);
}

// the penalty patch of entries e0 .. e0+15 (values in yv); KNOWN: the
// caller has established that the row has a history (which otherwise costs
// two dependent global loads per call)
template <int DT, bool KNOWN = false>
__device__ void patch16(const KParams& P, const RSmem& S, int row, int e0, float (&yv)[kEPT]) {
  if (!KNOWN && !row_has_penalty(P, row)) return;
  auto patch = [&](int li, float m, float a) {
#pragma unroll
    for (int j = 0; j < kEPT; ++j)
      if (j == li) yv[j] = penalise<DT>(yv[j], m, a);
  };
  if (S.pen_ok) {
    // entries e0 .. e0+15 lie in one slice: its bucket of the history
    const int sl = e0 / kWS, o0 = e0 % kWS;
    for (int i = S.poff[sl]; i < S.poff[sl + 1]; ++i) {
      const uint2 e = S.pent[i];
      const int li = static_cast<int>(e.x & 0xFFFFu) - o0;
      if (li >= 0 && li < kEPT) patch(li, DType<DT>::to_f32(e.x >> 16), __uint_as_float(e.y));
    }
    return;
  }
  const int slot = P.row_slot[row];
  const int len = min(P.slot_len[slot], P.hist_cap);
  const float rf = P.rep_factor ? P.rep_factor[row] : 1.0f;
  const long long hb = static_cast<long long>(slot) * P.hist_cap;
  for (int h = 0; h < len; ++h) {
    const int li = P.hist_tok[hb + h] - P.vocab_offset - e0;
    const int cn = P.hist_cnt[hb + h];
    if (cn <= 0 || li < 0 || li >= kEPT || e0 + li >= P.V) continue;
    patch(li, P.hist_mval ? P.hist_mval[hb + h] : penalty_divisor<DT>(cn, rf), additive_term(P, row, cn));
  }
}

// entries e0 .. e0+15 of the row read from global memory with the
// repetition-penalty patch applied (NaN past the row end)
template <int DT>
__device__ void load16(const KParams& P, const RSmem& S, int row, int e0, float (&yv)[kEPT]) {
  const uint16_t* src = static_cast<const uint16_t*>(P.logits) + logits_row_offset(P, row);
#pragma unroll
  for (int j = 0; j < kEPT; ++j) yv[j] = (e0 + j < P.V) ? DType<DT>::to_f32(src[e0 + j]) : __int_as_float(0x7FC00000);
  patch16<DT>(P, S, row, e0, yv);
}

// The raw word of entry e of the row with the penalty patch applied (one
// lane's share of a chunk that a warp reads entry by entry).
template <int DT>
__device__ uint32_t patched_raw(const KParams& P, const RSmem& S, int row, int e) {
  const uint16_t* src = static_cast<const uint16_t*>(P.logits) + logits_row_offset(P, row);
  const uint32_t raw = src[e];
  if (!row_has_penalty(P, row)) return raw;
  float y = DType<DT>::to_f32(raw);
  if (S.pen_ok) {
    const int sl = e / kWS, o = e % kWS;
    for (int i = S.poff[sl]; i < S.poff[sl + 1]; ++i) {
      const uint2 en = S.pent[i];
      if (static_cast<int>(en.x & 0xFFFFu) == o) y = penalise<DT>(y, DType<DT>::to_f32(en.x >> 16), __uint_as_float(en.y));
    }
  } else {
    const int slot = P.row_slot[row];
    const int len = min(P.slot_len[slot], P.hist_cap);
    const float rf = P.rep_factor ? P.rep_factor[row] : 1.0f;
    const long long hb = static_cast<long long>(slot) * P.hist_cap;
    for (int h = 0; h < len; ++h) {
      const int cn = P.hist_cnt[hb + h];
      if (cn > 0 && P.hist_tok[hb + h] - P.vocab_offset == e)
        y = penalise<DT>(y, P.hist_mval ? P.hist_mval[hb + h] : penalty_divisor<DT>(cn, rf), additive_term(P, row, cn));
    }
  }
  return DType<DT>::to_raw(y);
}

// The raw words of entries e0 .. e0+15 (e0 a multiple of 16): two 16-byte
// loads through L2, where a row just streamed still is, when the entries
// are whole and aligned; else 16 loads, with 0xFFFF (key 0) past the row end.
__device__ __forceinline__ void chunk_raw(const KParams& P, int row, int e0, uint4& a, uint4& b) {
  const uint16_t* src = static_cast<const uint16_t*>(P.logits) + logits_row_offset(P, row) + e0;
  if (P.vec_ok && e0 + kEPT <= P.V) {
    const uint4* g = reinterpret_cast<const uint4*>(src);
    a = __ldcg(g);
    b = __ldcg(g + 1);
  } else {
    uint32_t wv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t lo = (e0 + 2 * j < P.V) ? static_cast<uint32_t>(src[2 * j]) : 0xFFFFu;
      const uint32_t hi = (e0 + 2 * j + 1 < P.V) ? static_cast<uint32_t>(src[2 * j + 1]) : 0xFFFFu;
      wv[j] = lo | (hi << 16);
    }
    a = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    b = make_uint4(wv[4], wv[5], wv[6], wv[7]);
  }
}

// Streams rounds [r0, r1) of the row through the per-warp pipelines and calls
// fn(r, st, raw, w, nv) once per round with the warp's stage (its slice) and
// the thread's raw words and keys (nv of its 16 entries are in the row; the
// rest are padding, key 0).  Warps run through the rounds independently: fn
// may use block barriers only where every warp reaches them in the same
// round.  The next rounds are in flight while fn runs; the stage stays intact
// until fn returns.  Ends with a block barrier.
template <int DT, typename Fn>
__device__ void stream_row(const KParams& P, RSmem& S, int row, int r0, int r1, Fn&& fn) {
  const int R = (P.V + kRound - 1) / kRound;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool pen = row_has_penalty(P, row);
  const bool vec = P.vec_ok != 0;
  // rounds that need completing: all (unaligned rows, penalties), else a ragged last one
  const int rc = (!vec || pen) ? r0 : ((P.V % kRound) ? R - 1 : R);
  // this thread's chunks: the warp's slice of round r starts at chunk
  // r * kRVecs + warp * kWV; lane l copies chunks l and l + 32 of it
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(P.logits) +
                                                    logits_row_offset(P, row)) +
                     warp * kWV + lane;
  uint4* wst = &S.stage[0][0] + warp * (kStages * kWV);   // this warp's stages
  const int last_nv = max(0, min(kEPT, round_len(P.V, R - 1) - kEPT * static_cast<int>(threadIdx.x)));
  auto issue = [&](int x) {
    if (!vec) return;
    uint4* d = wst + (x % kStages) * kWV + lane;
    const uint4* g = src + static_cast<long long>(x) * kRVecs;
    if (x < R - 1) {   // whole slices
      cp_async16(d, g);
      cp_async16(d + 32, g + 32);
    } else {
      const int nfull = slice_len(P.V, x) >> 3;
      if (lane < nfull) cp_async16(d, g);
      if (lane + 32 < nfull) cp_async16(d + 32, g + 32);
    }
  };
  __syncthreads();  // the stages may have served as finishing scratch
  for (int s = 0; s < kStages - 1; ++s) {
    if (r0 + s < r1) issue(r0 + s);
    cp_async_commit();
  }
  for (int r = r0; r < r1; ++r) {
    cp_async_wait_group<kStages - 2>();
    // the slice of round r landed for the warp, and the warp is done with
    // round r - 1, whose stage the next copy reuses
    __syncwarp();
    uint4* st = wst + (r % kStages) * kWV;
    if (r >= rc) complete_slice<DT>(P, S, st, row, r, pen);
    uint32_t raw[8], w[8];
    round_load(st, raw, w);
    if (r + kStages - 1 < r1) issue(r + kStages - 1);
    cp_async_commit();
    fn(r, static_cast<const uint4*>(st), raw, w, (r < R - 1) ? kEPT : last_nv);
  }
  cp_async_wait_group<0>();
  __syncthreads();
}

// -------------------------------------------------------------- selection
// Lane-private 256-bin counts (S.lp) -> S.h256.  Barriers on both sides.
__device__ __forceinline__ void lp_zero(RSmem& S) {
  uint4* p = reinterpret_cast<uint4*>(S.lp);
  for (int i = threadIdx.x; i < 256 * 32 / 4; i += kT) p[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
}
__device__ __forceinline__ void lp_reduce(RSmem& S) {
  __syncthreads();
  const int t = threadIdx.x;
  if (t < 256) {
    unsigned acc = 0u;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) acc += S.lp[(t << 5) | ((j + t) & 31)];
    S.h256[t] = acc;
  }
  __syncthreads();
}

// Among bins 255..0 (descending), the first whose running count reaches n;
// -1 if the total stays below n.  *above = count of the bins above it.
// Warp 0 computes, everyone gets the result (barrier inside).
__device__ __forceinline__ int h256_select_desc(RSmem& S, unsigned n, unsigned* above) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    unsigned v[8], s = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) { v[j] = S.h256[255 - (lane * 8 + j)]; s += v[j]; }
    unsigned incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, incl >= n);
    int bin = -1;
    unsigned ab = 0u;
    if (hit) {
      const int L = __ffs(hit) - 1;
      if (lane == L) {
        unsigned acc = incl - s;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (bin < 0 && acc + v[j] >= n) { bin = 255 - (lane * 8 + j); ab = acc; }
          acc += v[j];
        }
      }
      bin = __shfl_sync(0xFFFFFFFFu, bin, L);
      ab = __shfl_sync(0xFFFFFFFFu, ab, L);
    }
    if (lane == 0) { S.ib[14] = bin; S.ib[15] = static_cast<int>(ab); }
  }
  __syncthreads();
  *above = static_cast<unsigned>(S.ib[15]);
  return S.ib[14];
}

// Among bins 0..nb-1 (ascending), the first whose running count reaches n;
// -1 if the total stays below n.  *above = count of the bins before it.
__device__ __forceinline__ int h256_select_asc(RSmem& S, unsigned n, unsigned* above) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    unsigned v[8], s = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) { v[j] = S.h256[lane * 8 + j]; s += v[j]; }
    unsigned incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, incl >= n);
    int bin = -1;
    unsigned ab = 0u;
    if (hit) {
      const int L = __ffs(hit) - 1;
      if (lane == L) {
        unsigned acc = incl - s;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (bin < 0 && acc + v[j] >= n) { bin = lane * 8 + j; ab = acc; }
          acc += v[j];
        }
      }
      bin = __shfl_sync(0xFFFFFFFFu, bin, L);
      ab = __shfl_sync(0xFFFFFFFFu, ab, L);
    }
    if (lane == 0) { S.ib[14] = bin; S.ib[15] = static_cast<int>(ab); }
  }
  __syncthreads();
  *above = static_cast<unsigned>(S.ib[15]);
  return S.ib[14];
}

// what one part of a split row hands to the part that finishes the row
struct PartHdr {
  unsigned kmax, first, floor, fill, overflow, pad0, pad1, pad2;
};

// ------------------------------------------------------- per-warp candidates
// Warp w keeps its candidates in region [w kCBW, (w + 1) kCBW) of the buffer,
// in vocab order; after the stream the regions are gathered into one buffer
// in vocab order.
constexpr int kCBW = kCB / kNW;           // 256
// After the stream the stages hold the gathered candidates (keys and
// indices of up to kCB: 48 KB) and, past them, the finishing histogram.
constexpr int kCntOff = 16384;            // words (64 KB)
__device__ __forceinline__ uint16_t* gkey(RSmem& S) { return reinterpret_cast<uint16_t*>(&S.stage[0][0]); }
__device__ __forceinline__ uint32_t* gidx(RSmem& S) { return reinterpret_cast<uint32_t*>(gkey(S) + kCB); }
constexpr int kKeepW = kCBW / 2;          // a compaction keeps about this many

// Among bins 0..255 (ascending, 8 per lane) of the warp-private histogram h,
// the first whose running count reaches n; -1 if the total stays below n.
// *above = count of the bins before it.  Warp-uniform result.
__device__ __forceinline__ int warp_sel_asc(const unsigned* h, unsigned n, unsigned* above) {
  const int lane = threadIdx.x & 31;
  unsigned v[8], s = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j) { v[j] = h[lane * 8 + j]; s += v[j]; }
  unsigned incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  const unsigned hit = __ballot_sync(0xFFFFFFFFu, incl >= n);
  if (!hit) { *above = __shfl_sync(0xFFFFFFFFu, incl, 31); return -1; }
  const int L = __ffs(hit) - 1;
  int bin = 0;
  unsigned ab = 0u;
  if (lane == L) {
    unsigned acc = incl - s;
    bin = -1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (bin < 0 && acc + v[j] >= n) { bin = lane * 8 + j; ab = acc; }
      acc += v[j];
    }
  }
  bin = __shfl_sync(0xFFFFFFFFu, bin, L);
  *above = __shfl_sync(0xFFFFFFFFu, ab, L);
  return bin;
}

// N-th largest key among the warp's region [0, fill) and this round's entries
// with key >= f (N <= their number); kref >= every one of those keys.  Bins
// are measured down from kref: 256 bins of 2^s keys give the lowest key of
// the bin where N is reached (a floor keeping at least N); only when that
// floor would not rise above f are the 2^s keys of the bin counted one by one.
__device__ unsigned wcand_nth(RSmem& S, int fill, const uint32_t (&w)[8], int nv, unsigned f, unsigned kref,
                              unsigned N) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned* h = S.lp + warp * 256;
  const uint16_t* ck = S.ckey + warp * kCBW;
  int sh = 0;
  while (((kref - f) >> sh) >= 256u) ++sh;
  for (int i = lane; i < 256; i += 32) h[i] = 0u;
  __syncwarp();
  for (int i = lane; i < fill; i += 32) {
    const unsigned key = ck[i];
    if (key >= f) atomicAdd(&h[(kref - key) >> sh], 1u);
  }
#pragma unroll
  for (int j = 0; j < kEPT; ++j) {
    const uint32_t key = ECAH_RKEY(w, j);
    if (j < nv && key >= f) atomicAdd(&h[(kref - key) >> sh], 1u);
  }
  __syncwarp();
  unsigned above;
  const int b1 = warp_sel_asc(h, N, &above);
  __syncwarp();
  if (sh == 0 || b1 < 0) return kref - static_cast<unsigned>(max(b1, 0));
  // the lowest key of bin b1 keeps at least N (and the whole bin) when it lies above f
  const unsigned span = (static_cast<unsigned>(b1) << sh) + ((1u << sh) - 1u);
  if (kref >= span && kref - span > f) return kref - span;
  const unsigned msk = (1u << sh) - 1u;
  for (int i = lane; i < 256; i += 32) h[i] = 0u;
  __syncwarp();
  for (int i = lane; i < fill; i += 32) {
    const unsigned d = kref - ck[i];
    if (ck[i] >= f && static_cast<int>(d >> sh) == b1) atomicAdd(&h[d & msk], 1u);
  }
#pragma unroll
  for (int j = 0; j < kEPT; ++j) {
    const uint32_t key = ECAH_RKEY(w, j);
    const unsigned d = kref - key;
    if (j < nv && key >= f && static_cast<int>(d >> sh) == b1) atomicAdd(&h[d & msk], 1u);
  }
  __syncwarp();
  unsigned ab2;
  const int b2 = warp_sel_asc(h, N - above, &ab2);
  __syncwarp();
  return kref - ((static_cast<unsigned>(b1) << sh) + static_cast<unsigned>(max(b2, 0)));
}

// keep the warp region's entries with key >= f, in order; returns the new fill
__device__ int wcand_compact(RSmem& S, int fill, unsigned f) {
  const int lane = threadIdx.x & 31, base = (threadIdx.x >> 5) * kCBW;
  uint16_t k[8];
  uint32_t ix[8];
  int cnt = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = lane * 8 + j;
    const bool in = i < fill;
    k[j] = in ? S.ckey[base + i] : 0;
    ix[j] = in ? S.cidx[base + i] : 0u;
    cnt += (in && k[j] >= f) ? 1 : 0;
  }
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  const int tot = __shfl_sync(0xFFFFFFFFu, incl, 31);
  __syncwarp();  // every lane has read its entries before they are overwritten
  int o = base + incl - cnt;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (lane * 8 + j < fill && k[j] >= f) { S.ckey[o] = k[j]; S.cidx[o] = ix[j]; ++o; }
  }
  __syncwarp();
  return tot;
}

// Gathers the warps' regions into one buffer [0, total) in vocab order
// (round, then warp, then position) in the stages (gkey / gidx below);
// returns total.  Every thread calls it; fill is the calling warp's region
// fill.
__device__ int gather_candidates(RSmem& S, int fill, int& ph) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned* cnt = S.lp;             // [warp][round] counts
  unsigned* obase = S.lp + 1024;    // [warp][round] output offsets
  unsigned* rstart = S.lp + 2048;   // [warp][round] first region slot of the round
  cnt[warp * 32 + lane] = 0u;
  __syncwarp();
  for (int i = lane; i < fill; i += 32) atomicAdd(&cnt[warp * 32 + (S.cidx[warp * kCBW + i] / kRound)], 1u);
  __syncwarp();
  const unsigned c = cnt[warp * 32 + lane];
  unsigned incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  rstart[warp * 32 + lane] = incl - c;
  __syncthreads();
  // thread t <-> (round t / 32, warp t % 32): offsets in round-major order
  int total;
  const int off = rscan_i(static_cast<int>(cnt[(tid & 31) * 32 + (tid >> 5)]), S, ph, &total);
  obase[(tid & 31) * 32 + (tid >> 5)] = static_cast<unsigned>(off);
  __syncthreads();
  uint16_t* tk = gkey(S);
  uint32_t* ti = gidx(S);
  for (int i = lane; i < fill; i += 32) {
    const uint32_t ix = S.cidx[warp * kCBW + i];
    const int rr = static_cast<int>(ix / kRound);
    const unsigned pos = obase[warp * 32 + rr] + (static_cast<unsigned>(i) - rstart[warp * 32 + rr]);
    tk[pos] = S.ckey[warp * kCBW + i];
    ti[pos] = ix;
  }
  __syncthreads();
  return total;
}

// Rows split over PP CTAs: each part publishes its max, first index of it,
// floor, candidates and segment masses; the last part to arrive merges them
// (max, first, floor, fill, overflow, cand in m; candidates into the stages;
// segment masses into S) and returns true to finish the row.  No CTA waits
// on another.  Kept out of line: it runs once per part.
struct PartState {
  unsigned kmax, first, f;
  int fill;
  bool overflow, cand;
};

__device__ __noinline__ bool part_exchange(const KParams& P, RSmem& S, int row, int part, int PP, int r0, int r1,
                                           int R, int N, bool mass_all, int& ph, PartState& m) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned kmax = m.kmax, first = m.first, f = m.f;
  int fill = m.fill;
  bool overflow = m.overflow, cand = m.cand;
    // ---------------------------------------- rows split over PP CTAs
    // Each part publishes its max, first index of it, floor, candidates
    // and segment masses; the last part to arrive merges them and finishes
    // the row (no CTA waits on another).
    PartHdr* hdr = static_cast<PartHdr*>(P.part_hdr) + static_cast<size_t>(row) * PP;
    unsigned long long* pc = P.part_cand + (static_cast<size_t>(row) * PP + part) * kCB;
    float2* pseg = P.part_seg + static_cast<size_t>(row) * (kMaxRounds * kNW);
    if (cand)
      for (int i = tid; i < fill; i += kT)
        pc[i] = (static_cast<unsigned long long>(gkey(S)[i]) << 32) | gidx(S)[i];
    if (mass_all)
      for (int i = r0 * kNW + tid; i < r1 * kNW; i += kT) pseg[i] = make_float2(S.ss[i], S.sq[i]);
    if (tid == 0) {
      PartHdr h;
      h.kmax = kmax; h.first = first; h.floor = f; h.fill = static_cast<unsigned>(cand ? fill : 0);
      h.overflow = overflow ? 1u : 0u; h.pad0 = h.pad1 = h.pad2 = 0u;
      hdr[part] = h;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) S.ib[6] = (atomicAdd(P.part_arrive + row, 1u) == static_cast<unsigned>(PP - 1)) ? 1 : 0;
    __syncthreads();
    if (S.ib[6] == 0) return false;   // another part finishes the row
    __threadfence();
    if (tid == 0) P.part_arrive[row] = 0u;   // ready for the next launch
    // the parts in order (lane q of warp 0 reads part q's header): the row
    // max, the first index of it (in the first part holding it), the
    // highest floor, any overflow, and where each part's candidates start
    if (warp == 0) {
      const bool has = lane < PP;
      PartHdr h{};
      if (has) {
        h.kmax = __ldcg(&hdr[lane].kmax);
        h.first = __ldcg(&hdr[lane].first);
        h.floor = __ldcg(&hdr[lane].floor);
        h.fill = __ldcg(&hdr[lane].fill);
        h.overflow = __ldcg(&hdr[lane].overflow);
      }
      const unsigned km = __reduce_max_sync(0xFFFFFFFFu, has ? h.kmax : 0u);
      const unsigned at = __ballot_sync(0xFFFFFFFFu, has && h.kmax == km);
      const unsigned fl = __shfl_sync(0xFFFFFFFFu, h.first, __ffs(at) - 1);
      const unsigned fr = __reduce_max_sync(0xFFFFFFFFu, has ? h.floor : 0u);
      const unsigned ov = __reduce_or_sync(0xFFFFFFFFu, has ? h.overflow : 0u);
      unsigned incl = has ? h.fill : 0u;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      S.pend[lane] = incl;   // inclusive end of part lane's candidates
      if (lane == 0) { S.ib[7] = static_cast<int>(km); S.ib[8] = static_cast<int>(fl); S.ib[9] = static_cast<int>(fr); S.ib[10] = static_cast<int>(ov); }
    }
    __syncthreads();
    kmax = static_cast<unsigned>(S.ib[7]);
    first = static_cast<unsigned>(S.ib[8]);
    if (N > 0) { f = static_cast<unsigned>(S.ib[9]); overflow = S.ib[10] != 0; }
    cand = N > 0 && !overflow;
    if (cand) {
      // every part's candidates with key >= f, in vocab order: thread t
      // takes 8 consecutive entries of the parts' concatenated lists per pass
      const int total = static_cast<int>(S.pend[PP - 1]);
      int base = 0;
      for (int g0 = 0; g0 < total && base <= kCB; g0 += kT * 8) {
        // addresses first (the part boundary is walked once per thread),
        // then all 8 loads in flight together, then the filter
        const unsigned long long* src[8];
        int g = g0 + tid * 8, q = 0;
        while (q < PP - 1 && g < total && static_cast<int>(S.pend[q]) <= g) ++q;
#pragma unroll
        for (int j = 0; j < 8; ++j, ++g) {
          src[j] = nullptr;
          if (g < total) {
            while (static_cast<int>(S.pend[q]) <= g) ++q;   // the part holding position g
            const int start = q ? static_cast<int>(S.pend[q - 1]) : 0;
            src[j] = P.part_cand + (static_cast<size_t>(row) * PP + q) * kCB + (g - start);
          }
        }
        unsigned long long e8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) e8[j] = src[j] ? __ldcg(src[j]) : 0ull;
        int c = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (static_cast<unsigned>(e8[j] >> 32) >= f) ++c;
          else e8[j] = 0ull;
        }
        int tot;
        int o = base + rscan_i(c, S, ph, &tot);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (e8[j] != 0ull) {   // key >= f >= 1, never a zero word
            if (o < kCB) {
              gkey(S)[o] = static_cast<uint16_t>(e8[j] >> 32);
              gidx(S)[o] = static_cast<uint32_t>(e8[j]);
            }
            ++o;
          }
        }
        base += tot;
      }
      if (base > kCB) {
        overflow = true;
        cand = false;
      } else {
        fill = base;
      }
    }
    if (mass_all)
      for (int i = tid; i < R * kNW; i += kT) {
        const int rr = i / kNW;
        if (rr < r0 || rr >= r1) {
          const float2 v = __ldcg(&pseg[i]);
          S.ss[i] = v.x;
          S.sq[i] = v.y;
        }
      }
    __syncthreads();
  m.kmax = kmax; m.first = first; m.f = f; m.fill = fill; m.overflow = overflow; m.cand = cand;
  return true;
}

// ------------------------------------------------------ per-round helpers
// packed fp32 pairs (sm_100 f32x2 ALU operations, round to nearest)
__device__ __forceinline__ unsigned long long pk(float2 a) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
  return r;
}
__device__ __forceinline__ float2 upk(unsigned long long r) {
  float2 a;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(r));
  return a;
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)), "l"(pk(c)));
  return upk(r);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)));
  return upk(r);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)));
  return upk(r);
}

// Sum over a thread's 16 entries of 2^(z log2e - c), z = y / T rounded as
// the IEEE divide (reciprocal, residual and correction, as mass_of) or y
// itself at T == 1; one rounding in the exponent.  GUARD drops NaN masses
// (padding of a ragged last round).
template <int DT, bool T1, bool GUARD>
__device__ __forceinline__ float seg_masses(const uint32_t (&raw)[8], float T, float rT, float c) {
  const float2 L2 = make_float2(kLog2e, kLog2e), nc2 = make_float2(-c, -c);
  const float2 rT2 = make_float2(rT, rT), nT2 = make_float2(-T, -T);
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 y = vals2<DT>(raw[j]);
    float2 z = y;
    if (!T1) {
      const float2 q = fmul2(y, rT2);
      z = ffma2(ffma2(q, nT2, y), rT2, q);
    }
    const float2 a = ffma2(z, L2, nc2);
    float2 e = make_float2(ex2_approx(a.x), ex2_approx(a.y));
    if (GUARD) e = make_float2(fmaxf(e.x, 0.f), fmaxf(e.y, 0.f));
    acc = fadd2(acc, e);
  }
  return acc.x + acc.y;
}

// mass_of(y, T, rT, M) of a thread's 16 entries (entry j in e[j]), two at a
// time with the same roundings: q = y rT, z = q + rT (y - q T), then
// 2^((z - M) log2e).  Padding entries (NaN) give NaN.
template <int DT>
__device__ __forceinline__ void masses16(const uint32_t (&raw)[8], float T, float rT, float M, float (&e)[kEPT]) {
  const float2 rT2 = make_float2(rT, rT), nT2 = make_float2(-T, -T);
  const float2 nM2 = make_float2(-M, -M), L2 = make_float2(kLog2e, kLog2e);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 y = vals2<DT>(raw[j]);
    const float2 q = fmul2(y, rT2);
    const float2 z = ffma2(ffma2(q, nT2, y), rT2, q);
    const float2 d = fmul2(fadd2(z, nM2), L2);
    e[2 * j] = ex2_approx(d.x);
    e[2 * j + 1] = ex2_approx(d.y);
  }
}

// mass of an entry relative to reference q (scaled like z): mass_of with
// the T == 1 shortcut (z = y exactly, as the divide gives)
__device__ __forceinline__ float emass(float y, float T, float rT, float q, bool t1) {
  return t1 ? ex2_approx(__fmul_rn(__fsub_rn(y, q), kLog2e)) : mass_of(y, T, rT, q);
}

// Reference of a segment whose sum is already relative to the row max M
// (masses from mass_of): rescaling by 2^(RN(M log2e) - M log2e) would scale
// it by the rounding error of M log2e, which for large M (small T) is not
// negligible.
constexpr float kRelM = INFINITY;

// segment s's mass rescaled to M: ss 2^(c - M log2e), with the exponent
// rounded once (0 past nseg, for empty segments and for references far
// enough below M to underflow; NaN sums stay NaN; sums with reference kRelM
// as they are)
__device__ __forceinline__ float seg_mass(const RSmem& S, int s, int nseg, float M) {
  if (s >= nseg) return 0.f;
  const float ss = S.ss[s];
  if (ss != ss) return ss;
  const float q = S.sq[s];
  if (q == kRelM) return ss;
  return (ss > 0.f) ? __fmul_rn(ss, ex2_approx(__fmaf_rn(-M, kLog2e, q))) : 0.f;
}

// ------------------------------------------------------------ selection over the finish
// Among the finishing histogram's bins (bin b: key kmax - b, four per
// thread), the first whose running count reaches n; INT_MAX when the total
// stays below n.  *tot = the histogram's total.  Every thread gets the result.
__device__ __forceinline__ unsigned cnth_select(const unsigned* cnth, int n, RSmem& S, int& ph, int* tot) {
  const int tid = threadIdx.x;
  unsigned c4 = 0u;
#pragma unroll
  for (int j = 0; j < 4; ++j) c4 += cnth[tid * 4 + j];
  const int ex = rscan_i(static_cast<int>(c4), S, ph, tot);
  int mine = INT_MAX;
  if (static_cast<unsigned>(ex) < static_cast<unsigned>(n) && static_cast<unsigned>(ex) + c4 >= static_cast<unsigned>(n)) {
    unsigned acc = static_cast<unsigned>(ex);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const unsigned v = cnth[tid * 4 + j];
      if (mine == INT_MAX && acc + v >= static_cast<unsigned>(n)) mine = tid * 4 + j;
      acc += v;
    }
  }
  return rmin_u(static_cast<unsigned>(mine), S, ph);
}

// The k-th largest key of the row (1 <= k <= its length) by a two-digit
// (8 | 8 bit) radix select over two re-streams.  Every thread gets it.
template <int DT>
__device__ uint32_t radix_kth(const KParams& P, RSmem& S, int row, int R, unsigned k) {
  const uint32_t lane = threadIdx.x & 31;
  lp_zero(S);
  stream_row<DT>(P, S, row, 0, R, [&](int, const uint4*, uint32_t (&)[8], uint32_t (&w)[8], int nv) {
#pragma unroll
    for (int j = 0; j < kEPT; ++j)
      if (j < nv) atomicAdd(&S.lp[((ECAH_RKEY(w, j) >> 8) << 5) | lane], 1u);
  });
  lp_reduce(S);
  unsigned above;
  const int hb = h256_select_desc(S, k, &above);
  lp_zero(S);
  stream_row<DT>(P, S, row, 0, R, [&](int, const uint4*, uint32_t (&)[8], uint32_t (&w)[8], int nv) {
#pragma unroll
    for (int j = 0; j < kEPT; ++j) {
      const uint32_t key = ECAH_RKEY(w, j);
      if (j < nv && static_cast<int>(key >> 8) == hb) atomicAdd(&S.lp[((key & 255u) << 5) | lane], 1u);
    }
  });
  lp_reduce(S);
  unsigned ab2;
  const int lb = h256_select_desc(S, k - above, &ab2);
  return (static_cast<uint32_t>(hb) << 8) | static_cast<uint32_t>(lb);
}

// ------------------------------------------------ rows finished from chunk records
// Unsplit top-k rows keep no candidates while streaming.  Instead, for every
// chunk of 16 entries (round r, thread t: entries r kRound + 16 t .. + 15,
// chunk index c = r kT + t) the stream records the chunk's top key, in the
// ckey and cidx regions (kRecRounds rounds at most).
constexpr int kRecRounds = kCB * (sizeof(uint16_t) + sizeof(uint32_t)) / sizeof(uint16_t) / kT;   // 24
static_assert(offsetof(RSmem, cidx) == offsetof(RSmem, ckey) + sizeof(RSmem::ckey), "records span ckey and cidx");
__device__ __forceinline__ uint16_t* recs(RSmem& S) { return S.ckey; }

// raw word j (0..15) of a chunk held as two uint4
__device__ __forceinline__ uint32_t raw_at(const uint4& a, const uint4& b, int j) {
  const uint32_t wv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t w = wv[0];
#pragma unroll
  for (int q = 1; q < 8; ++q)
    if ((j >> 1) == q) w = wv[q];
  return (j & 1) ? (w >> 16) : (w & 0xFFFFu);
}

struct LeanRes {
  bool ok;                     // false: nothing decided, the caller takes the re-streaming paths
  int result;
  float Z;
  uint32_t key_lo_k, key_lo, kdraw;
};

// The repetition-penalty patch of a chunk's 16 raw words (two uint4), as the
// stream applied it.
template <int DT>
__device__ __forceinline__ void patch_chunk(const KParams& P, const RSmem& S, int row, int e0, uint4& a, uint4& b) {
  uint32_t wv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float yv[kEPT];
#pragma unroll
  for (int j = 0; j < kEPT; ++j) yv[j] = DType<DT>::to_f32((j & 1) ? (wv[j >> 1] >> 16) : (wv[j >> 1] & 0xFFFFu));
  patch16<DT, true>(P, S, row, e0, yv);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t lo = (e0 + 2 * j < P.V) ? DType<DT>::to_raw(yv[2 * j]) : 0xFFFFu;
    const uint32_t hi = (e0 + 2 * j + 1 < P.V) ? DType<DT>::to_raw(yv[2 * j + 1]) : 0xFFFFu;
    wv[j] = lo | (hi << 16);
  }
  a = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  b = make_uint4(wv[4], wv[5], wv[6], wv[7]);
}

// bit j set where key j of the chunk is >= f (f >= 1: key 0, past the row
// end, never is)
__device__ __forceinline__ uint32_t chunk_mask(const uint4& a, const uint4& b, uint32_t f) {
  const uint32_t fm2 = (f - 1u) * 0x00010001u;
  const uint32_t wv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t m = 0u;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const uint32_t s2 = surv2(keys2(wv[q]), fm2);   // 1 in each half whose key >= f
    m |= ((s2 & 1u) | ((s2 >> 15) & 2u)) << (2 * q);
  }
  return m;
}

// Flagged chunks: a list in vocab order (in S.lp); item i's 16 entries, with
// the penalty patch applied, are cached in the stages from kLeanCacheOff on.
constexpr int kLeanCacheOff = kHB * 4 / 16;                       // uint4 index: after the counts
constexpr int kLeanCacheCap = (kStages * kRVecs - kLeanCacheOff) / 2;   // chunks (3584)

// Thresholds and draw of a record row.
//   1. A floor F that every kept entry reaches: the k-th largest of the
//      threads' largest records (k chunks hold an entry at or above it, so
//      the row's k-th largest key is not below it, and top-p acts on the
//      top-k set).  When the records do not place F within the 4096 keys
//      under the row max, F is the lowest key of that window.  Every entry
//      at or above F lies in a chunk whose top key is at or above F.
//   2. Those chunks, listed in vocab order and spread evenly over the
//      threads, are re-read (from L2) once and cached in shared memory; their
//      entries at or above F are counted per key: tau_k and tau_p as on the
//      candidate path.
//   3. Thread t holds list items [q t, q t + q), so thread order is vocab
//      order: per-thread kept masses, one block scan, and the thread holding
//      u Z walks its items to the drawn entry.
// Returns ok = false when a threshold falls below F (the window), the list
// outgrows the cache, or no kept entry has mass.
template <int DT>
__device__ __forceinline__ LeanRes lean_finish(const KParams& P, RSmem& S, int row, int R, uint32_t kmax, float M, float T,
                                            float rT, int k, bool topp, float pp, uint32_t key_cut, float u, int& ph) {
  using C = Codec<DT, 16>;
  const int tid = threadIdx.x;
  LeanRes res{false, 0, 0.f, 0u, 0u, 0u};
  const uint16_t* rec1 = recs(S);
  unsigned* cnt = reinterpret_cast<unsigned*>(&S.stage[0][0]);   // exact counts, bin b: key kmax - b
  unsigned* cf = cnt + kHB;                                       // counts of recorded keys (the floor)
  uint4* cache = &S.stage[0][0] + kLeanCacheOff;                  // overlaps cf: used after the floor
  uint16_t* list = reinterpret_cast<uint16_t*>(S.lp);
  const uint32_t klo = (kmax >= static_cast<uint32_t>(kHB)) ? kmax - static_cast<uint32_t>(kHB - 1) : 1u;
  for (int i = tid; i < kHB; i += kT) { cnt[i] = 0u; cf[i] = 0u; }
  __syncthreads();

  // ---- 1. the floor, from counts of the threads' largest records
  uint32_t km = 0u;
  for (int r = 0; r < R; ++r) km = max(km, static_cast<uint32_t>(rec1[r * kT + tid]));
  if (km >= klo) atomicAdd(&cf[kmax - km], 1u);
  __syncthreads();
  int ftot;
  const unsigned fb = cnth_select(cf, k, S, ph, &ftot);
  const uint32_t F = (ftot < k || fb == static_cast<unsigned>(INT_MAX)) ? klo : kmax - fb;

  // ---- 2. the flagged chunks in vocab order, read once
  const int nch = (P.V + kEPT - 1) / kEPT;
  const int c0 = tid * R, c1 = min(c0 + R, nch);
  int nf = 0;
  for (int c = c0; c < c1; ++c) nf += rec1[c] >= F ? 1 : 0;
  int n;
  int o = rscan_i(nf, S, ph, &n);
  if (n > kLeanCacheCap) return res;
  for (int c = c0; c < c1; ++c)
    if (rec1[c] >= F) list[o++] = static_cast<uint16_t>(c);
  __syncthreads();
  const int q = (n + kT - 1) / kT;
  const int i0 = min(tid * q, n), i1 = min(i0 + q, n);
  const bool pen = row_has_penalty(P, row);
  {
    // one chunk in flight while the previous one is counted
    uint4 na = make_uint4(0u, 0u, 0u, 0u), nb = na;
    if (i0 < i1) chunk_raw(P, row, static_cast<int>(list[i0]) * kEPT, na, nb);
    for (int i = i0; i < i1; ++i) {
      uint4 ca = na, cb = nb;
      if (i + 1 < i1) chunk_raw(P, row, static_cast<int>(list[i + 1]) * kEPT, na, nb);
      if (pen) patch_chunk<DT>(P, S, row, static_cast<int>(list[i]) * kEPT, ca, cb);
      for (uint32_t m = chunk_mask(ca, cb, F); m; m &= m - 1u)
        atomicAdd(&cnt[kmax - key16(raw_at(ca, cb, __ffs(m) - 1))], 1u);
      cache[2 * i] = ca;
      cache[2 * i + 1] = cb;
    }
  }
  __syncthreads();

  // ---- thresholds, as on the candidate path
  int ktot;
  const unsigned ksel = cnth_select(cnt, k, S, ph, &ktot);
  if (ktot < k || ksel == static_cast<unsigned>(INT_MAX)) return res;
  const uint32_t key_lo_k = tie_floor<DT, 16>(kmax - ksel, T);
  if (key_lo_k < F) return res;
  uint32_t key_lo = key_lo_k;
  if (topp) {
    const int bk = static_cast<int>(kmax - key_lo_k);
    float m4[4];
    float s4 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = tid * 4 + j;
      const unsigned cn = cnt[b];
      m4[j] = (b <= bk && cn) ? __fmul_rn(static_cast<float>(cn), mass_of(C::value(kmax - static_cast<uint32_t>(b)), T, rT, M)) : 0.f;
      s4 += m4[j];
    }
    float tot;
    const float ex = rscan_f(s4, S, ph, &tot);
    const float target = __fmul_rn(pp, tot);   // top-p over the top-k set
    int mine = INT_MAX;
    if (s4 > 0.f && ex + s4 >= target) {
      float acc = ex;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (mine == INT_MAX && m4[j] > 0.f && acc + m4[j] >= target) mine = tid * 4 + j;
        acc += m4[j];
      }
      if (mine == INT_MAX) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (m4[j] > 0.f) mine = tid * 4 + j;
      }
    }
    unsigned bsel = rmin_u(static_cast<unsigned>(mine), S, ph);
    const bool reached = tot >= target;
    if (bsel == static_cast<unsigned>(INT_MAX) && reached) {
      int last = -1;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (m4[j] > 0.f) last = tid * 4 + j;
      bsel = static_cast<unsigned>(static_cast<int>(rmax_u(static_cast<unsigned>(last + 1), S, ph)) - 1);
    }
    if (!reached || bsel == static_cast<unsigned>(INT_MAX) || bsel == 0xFFFFFFFFu) return res;
    key_lo = max(tie_floor<DT, 16>(kmax - bsel, T), key_lo_k);
    if (key_lo < F) return res;
  }
  const uint32_t kdraw = max(key_lo, key_cut);

  // ---- 3. the draw: kept masses per thread in vocab order
  float wsum = 0.f;
  for (int i = i0; i < i1; ++i) {
    const uint4 ca = cache[2 * i], cb = cache[2 * i + 1];
    for (uint32_t m = chunk_mask(ca, cb, kdraw); m; m &= m - 1u)
      wsum += mass_of(DType<DT>::to_f32(raw_at(ca, cb, __ffs(m) - 1)), T, rT, M);
  }
  float Z;
  const float ex = rscan_f(wsum, S, ph, &Z);
  const float target = __fmul_rn(u, Z);
  const unsigned mine = (wsum > 0.f && ex + wsum > target) ? static_cast<unsigned>(tid) : static_cast<unsigned>(INT_MAX);
  unsigned pick, lastp;
  rminmax_u(mine, wsum > 0.f ? static_cast<unsigned>(tid + 1) : 0u, S, ph, &pick, &lastp);
  if (pick == static_cast<unsigned>(INT_MAX) && lastp == 0u) return res;
  const bool take_last = pick == static_cast<unsigned>(INT_MAX);
  const int owner = take_last ? static_cast<int>(lastp) - 1 : static_cast<int>(pick);
  if (tid == owner) {
    // the same sums in the same order: ex + (running sum) crosses the target
    // inside this thread's items, or the last kept entry is taken
    float run = 0.f;
    int hit = -1, lastk = -1;
    for (int i = i0; i < i1 && hit < 0; ++i) {
      const uint4 ca = cache[2 * i], cb = cache[2 * i + 1];
      const int e0 = static_cast<int>(list[i]) * kEPT;
      for (uint32_t m = chunk_mask(ca, cb, kdraw); m && hit < 0; m &= m - 1u) {
        const int j = __ffs(m) - 1;
        run += mass_of(DType<DT>::to_f32(raw_at(ca, cb, j)), T, rT, M);
        lastk = e0 + j;
        if (!take_last && ex + run > target) hit = e0 + j;
      }
    }
    S.ib[4] = hit >= 0 ? hit : lastk;
  }
  __syncthreads();
  res.ok = S.ib[4] >= 0;
  res.result = S.ib[4];
  res.Z = Z;
  res.key_lo_k = key_lo_k;
  res.key_lo = key_lo;
  res.kdraw = kdraw;
  return res;
}

// ------------------------------------------------ top-p rows finished from chunk records
// Unsplit rows with top-p and no top-k keep no candidates while streaming.
// For every chunk of 16 entries the stream records its two largest keys
// (top1 | top2 << 16; chunk c = r kT + t as for top-k records), in the ckey
// and cidx regions, while it sums the row's masses per segment as usual.
constexpr int kRec2Rounds = kCB * (sizeof(uint16_t) + sizeof(uint32_t)) / sizeof(uint32_t) / kT;   // 12
__device__ __forceinline__ uint32_t* recs2(RSmem& S) { return reinterpret_cast<uint32_t*>(S.ckey); }

// The two largest of a thread's 16 keys (8 packed words, 2 keys each) as
// top1 | top2 << 16.  Each half runs a tournament keeping its two largest
// (the second of a merge of sorted pairs (a1 >= a2), (b1 >= b2) is
// max(min(a1, b1), max(a2, b2))), then the halves merge the same way.
__device__ __forceinline__ uint32_t top2_16(const uint32_t (&w)[8]) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    h[q] = max16x2(w[2 * q], w[2 * q + 1]);
    l[q] = min16x2(w[2 * q], w[2 * q + 1]);
  }
  const uint32_t H01 = max16x2(h[0], h[1]), L01 = max16x2(min16x2(h[0], h[1]), max16x2(l[0], l[1]));
  const uint32_t H23 = max16x2(h[2], h[3]), L23 = max16x2(min16x2(h[2], h[3]), max16x2(l[2], l[3]));
  const uint32_t H = max16x2(H01, H23), L = max16x2(min16x2(H01, H23), max16x2(L01, L23));
  const uint32_t a1 = H & 0xFFFFu, b1 = H >> 16, a2 = L & 0xFFFFu, b2 = L >> 16;
  return max(a1, b1) | (max(min(a1, b1), max(a2, b2)) << 16);
}

// The first bin b (four per thread, bin 4 tid + j) where the running sum of
// m4 over bins in order reaches target, given this thread's exclusive prefix
// ex and the block total tot.  When rounding keeps every thread's running sum
// short although tot reaches the target, the last non-zero bin.  INT_MAX
// when tot stays below the target.  Every thread gets the result.
__device__ __forceinline__ int cross_bin(const float (&m4)[4], float s4, float ex, float tot, float target, RSmem& S,
                                         int& ph) {
  const int tid = threadIdx.x;
  int mine = INT_MAX;
  if (s4 > 0.f && ex + s4 >= target) {
    float acc = ex;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (mine == INT_MAX && m4[j] > 0.f && acc + m4[j] >= target) mine = tid * 4 + j;
      acc += m4[j];
    }
    if (mine == INT_MAX) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (m4[j] > 0.f) mine = tid * 4 + j;
    }
  }
  unsigned bsel = rmin_u(static_cast<unsigned>(mine), S, ph);
  if (bsel == static_cast<unsigned>(INT_MAX) && tot >= target) {
    int last = -1;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (m4[j] > 0.f) last = tid * 4 + j;
    bsel = static_cast<unsigned>(static_cast<int>(rmax_u(static_cast<unsigned>(last + 1), S, ph)) - 1);
  }
  if (tot < target || bsel == 0xFFFFFFFFu) return INT_MAX;
  return static_cast<int>(bsel);
}

// The records' counts per key live in S.lp, a histogram of kPleanNB bins that
// the stream fills as it records: bin h holds key hwhi - h, where hwhi is
// round 0's max plus kPleanHead (the row max is almost always within that
// headroom; when it is not, the finish histograms the records again).
constexpr int kPleanHead = 512;
constexpr int kPleanNB = kHB + kPleanHead;

// counts a thread's two records (top1 | top2 << 16) into the histogram
__device__ __forceinline__ void plean_count(RSmem& S, uint32_t t12, uint32_t hwhi) {
  const uint32_t t1 = t12 & 0xFFFFu, t2 = t12 >> 16;
  const uint32_t d1 = hwhi - t1, d2 = hwhi - t2;   // keys above hwhi wrap past the bins
  if (d1 < static_cast<uint32_t>(kPleanNB) && t1 != 0u) atomicAdd(&S.lp[d1], 1u);
  if (d2 < static_cast<uint32_t>(kPleanNB) && t2 != 0u) atomicAdd(&S.lp[d2], 1u);
}

// Finish scratch in the stages (after the stream), in 4-byte words: the mass
// of each of the 4096 keys under the row max, then (sized once the count n of
// re-read chunks is known) the list of those chunks, their kept masses and a
// cache of their 16 entries.
constexpr int kPleanListOff = kHB;                      // words
constexpr int kStageWords = kStages * kRVecs * 4;

// Top-p threshold and draw of a record row, without re-streaming it.
//   1. The records alone bound the mass at or above each key from below:
//      every record is an entry.  bL = the first bin where that lower bound
//      reaches p S; the kept set's lowest key tau_p is then at or above
//      v = kmax - bL.
//   2. An entry at or above v that is not a record lies in a chunk whose
//      top2 is at or above v.  Those chunks (listed in vocab order) are
//      copied into shared memory, all copies in flight at once (from L2
//      where the row still is): their entries at or
//      above v are added to the histogram and their two records taken out,
//      which leaves exact counts in every bin up to bL (any other chunk's
//      entries at or above v are its top1 alone).
//   3. tau_p from those exact counts, as on the candidate path; then each
//      re-read chunk's kept mass.
//   4. The draw in vocab order: thread t owns chunks [R t, R t + R); a
//      re-read chunk contributes its kept mass, any other its top1 when kept.
//      The thread holding u Z finds the chunk where the running sum crosses
//      u Z, and warp 0 reads that chunk entry by entry (a top1 is unique in
//      its chunk, or the chunk's top2 would equal it and the chunk would have
//      been re-read).
// The per-bin masses of the bound and of the exact counts are summed in the
// same order, and an exact count is never below the records' count of its
// bin, so the exact running sum reaches p S no later than bin bL.  Returns
// ok = false (nothing decided) when the bound does not reach p S within the
// window, the listed chunks outgrow the shared-memory cache (a wide
// nucleus), or tau_p lands below v after the tie floor.
template <int DT>
__device__ __forceinline__ LeanRes plean_finish(const KParams& P, RSmem& S, int row, int R, uint32_t kmax, float M,
                                             float T, float rT, float pp, float S_all, uint32_t key_cut, float u,
                                             uint32_t hwhi, int& ph) {
  using C = Codec<DT, 16>;
  const int tid = threadIdx.x;
  LeanRes res{false, 0, 0.f, 0u, 0u, 0u};
  const uint32_t* rec = recs2(S);
  unsigned* cL = S.lp;
  unsigned* sw = reinterpret_cast<unsigned*>(&S.stage[0][0]);
  float* mt = reinterpret_cast<float*>(sw);
  const uint32_t klo = (kmax >= static_cast<uint32_t>(kHB)) ? kmax - static_cast<uint32_t>(kHB - 1) : 1u;
  const int nch = (P.V + kEPT - 1) / kEPT;

  // bin b (key kmax - b) of the histogram is cL[b + hoff]
  uint32_t hoff = hwhi - kmax;
  if (kmax > hwhi) {
    // the row max lies above the stream's window: count the records again
    for (int i = tid; i < kPleanNB; i += kT) cL[i] = 0u;
    __syncthreads();
    for (int r = 0; r < R; ++r) {
      const uint32_t rv = rec[r * kT + tid];
      const uint32_t t1 = rv & 0xFFFFu, t2 = rv >> 16;
      if (t1 >= klo) atomicAdd(&cL[kmax - t1], 1u);
      if (t2 >= klo) atomicAdd(&cL[kmax - t2], 1u);
    }
    hoff = 0u;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int b = tid * 4 + j;
    mt[b] = (kmax - static_cast<uint32_t>(b) >= klo && kmax >= static_cast<uint32_t>(b))
                ? mass_of(C::value(kmax - static_cast<uint32_t>(b)), T, rT, M) : 0.f;
  }
  __syncthreads();

  // ---- 1. the records' lower bound
  const float target = __fmul_rn(pp, S_all);
  float m4[4];
  float s4 = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int b = tid * 4 + j;
    m4[j] = __fmul_rn(static_cast<float>(cL[b + hoff]), mt[b]);
    s4 += m4[j];
  }
  float tot;
  float ex = rscan_f(s4, S, ph, &tot);
  const int bL = cross_bin(m4, s4, ex, tot, target, S, ph);
  if (bL == INT_MAX) return res;
  const uint32_t v = kmax - static_cast<uint32_t>(bL);

  // ---- 2. chunks that may hold unrecorded entries at or above v
  const int c0 = tid * R, c1 = min(c0 + R, nch);
  int nf = 0;
  for (int c = c0; c < c1; ++c) nf += (rec[c] >> 16) >= v ? 1 : 0;
  int n;
  const int o0 = rscan_i(nf, S, ph, &n);
  uint16_t* list = reinterpret_cast<uint16_t*>(sw + kPleanListOff);
  float* imass = reinterpret_cast<float*>(sw + kPleanListOff + ((n + 7) / 8) * 4);
  uint4* cache = reinterpret_cast<uint4*>(sw + kPleanListOff + ((n + 7) / 8) * 4 + ((n + 3) / 4) * 4);
  // a nucleus so wide that its chunks outgrow the cache goes to the
  // re-streaming paths, which handle it at less cost than re-reading them
  if (n > (kStageWords - (kPleanListOff + ((n + 7) / 8) * 4 + ((n + 3) / 4) * 4)) / 8) return res;
  {
    int o = o0;
    for (int c = c0; c < c1; ++c)
      if ((rec[c] >> 16) >= v) list[o++] = static_cast<uint16_t>(c);
  }
  __syncthreads();
  const bool pen = row_has_penalty(P, row);
  // the listed chunks come in through the cache, every thread's copies in
  // flight together; item i sits in slot i
  for (int i = tid; i < n; i += kT) {
    const int e0 = static_cast<int>(list[i]) * kEPT;
    uint4* d = cache + 2 * i;
    if (P.vec_ok && e0 + kEPT <= P.V) {
      const uint4* g = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(P.logits) + logits_row_offset(P, row) + e0);
      cp_async16(d, g);
      cp_async16(d + 1, g + 1);
    } else {
      chunk_raw(P, row, e0, d[0], d[1]);
    }
  }
  cp_async_wait_all();
  __syncthreads();
  for (int i = tid; i < n; i += kT) {
    uint4 ca = cache[2 * i], cb = cache[2 * i + 1];
    const int c = list[i];
    if (pen) {
      patch_chunk<DT>(P, S, row, c * kEPT, ca, cb);
      cache[2 * i] = ca;
      cache[2 * i + 1] = cb;
    }
    for (uint32_t m = chunk_mask(ca, cb, v); m; m &= m - 1u)
      atomicAdd(&cL[kmax - key16(raw_at(ca, cb, __ffs(m) - 1)) + hoff], 1u);
    const uint32_t rv = rec[c];
    atomicSub(&cL[kmax - (rv & 0xFFFFu) + hoff], 1u);
    atomicSub(&cL[kmax - (rv >> 16) + hoff], 1u);
  }
  __syncthreads();

  // ---- 3. tau_p from the exact counts of the bins at or above v
  s4 = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int b = tid * 4 + j;
    m4[j] = (b <= bL) ? __fmul_rn(static_cast<float>(cL[b + hoff]), mt[b]) : 0.f;
    s4 += m4[j];
  }
  ex = rscan_f(s4, S, ph, &tot);
  const int bs = cross_bin(m4, s4, ex, tot, target, S, ph);
  if (bs == INT_MAX) return res;
  const uint32_t key_lo = tie_floor<DT, 16>(kmax - static_cast<uint32_t>(bs), T);
  if (key_lo < v) return res;
  const uint32_t kdraw = max(key_lo, key_cut);
  // each listed chunk's kept mass, from the cache (patched)
  for (int i = tid; i < n; i += kT) {
    const uint4 ca = cache[2 * i], cb = cache[2 * i + 1];
    float sm = 0.f;
    for (uint32_t m = chunk_mask(ca, cb, kdraw); m; m &= m - 1u) sm += mt[kmax - key16(raw_at(ca, cb, __ffs(m) - 1))];
    imass[i] = sm;
  }
  __syncthreads();

  // ---- 4. the draw over this thread's chunks, in vocab order
  float wsum = 0.f;
  {
    int i = o0;
    for (int c = c0; c < c1; ++c) {
      const uint32_t rv = rec[c];
      if ((rv >> 16) >= v) wsum += imass[i++];
      else if ((rv & 0xFFFFu) >= kdraw) wsum += mt[kmax - (rv & 0xFFFFu)];
    }
  }
  float Z;
  ex = rscan_f(wsum, S, ph, &Z);
  const float tgt = __fmul_rn(u, Z);
  const unsigned mine = (wsum > 0.f && ex + wsum > tgt) ? static_cast<unsigned>(tid) : static_cast<unsigned>(INT_MAX);
  unsigned pick, lastp;
  rminmax_u(mine, wsum > 0.f ? static_cast<unsigned>(tid + 1) : 0u, S, ph, &pick, &lastp);
  if (pick == static_cast<unsigned>(INT_MAX) && lastp == 0u) return res;
  const bool take_last = pick == static_cast<unsigned>(INT_MAX);
  const int owner = take_last ? static_cast<int>(lastp) - 1 : static_cast<int>(pick);
  if (tid == owner) {
    // the same sums in the same order: the chunk where ex + (running sum)
    // crosses the target, or the last with kept mass
    float run = ex, base = ex;
    int hc = -1, hi = -1, i = o0;
    for (int c = c0; c < c1; ++c) {
      const uint32_t rv = rec[c];
      float add = 0.f;
      int ii = -1;
      if ((rv >> 16) >= v) { ii = i++; add = imass[ii]; }
      else if ((rv & 0xFFFFu) >= kdraw) add = mt[kmax - (rv & 0xFFFFu)];
      if (add > 0.f) {
        hc = c; hi = ii; base = run;
        run += add;
        if (!take_last && run > tgt) break;
      }
    }
    S.ib[5] = hc;
    S.ib[6] = hi;
    S.fb[5] = base;
  }
  __syncthreads();
  if (tid < 32) {
    // warp 0 reads that chunk, one entry per lane: a re-read chunk's kept
    // masses summed over the lanes in order (its last kept entry when
    // rounding keeps the running sum short); a top1 located in its chunk
    const int hc = S.ib[5], hi = S.ib[6], lane = tid;
    int e = -1;
    if (hc >= 0) {
      const int ej = hc * kEPT + lane;
      uint32_t key = 0u;
      if (lane < kEPT && ej < P.V)
        key = key16(hi >= 0 ? static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(cache + 2 * hi)[lane])
                            : patched_raw<DT>(P, S, row, ej));
      if (hi >= 0) {
        const float m = (lane < kEPT && key >= kdraw) ? mt[kmax - key] : 0.f;
        float incl = m;
#pragma unroll
        for (int o = 1; o < kEPT; o <<= 1) {
          const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += y;
        }
        const unsigned hit = __ballot_sync(0xFFFFFFFFu, !take_last && m > 0.f && S.fb[5] + incl > tgt);
        const unsigned nz = __ballot_sync(0xFFFFFFFFu, m > 0.f);
        e = hc * kEPT + (hit ? __ffs(hit) - 1 : (nz ? 31 - __clz(nz) : 0));
      } else {
        const unsigned b = __ballot_sync(0xFFFFFFFFu, lane < kEPT && key == (rec[hc] & 0xFFFFu));
        e = hc * kEPT + (b ? __ffs(b) - 1 : 0);
      }
    }
    if (lane == 0) S.ib[4] = e;
  }
  __syncthreads();
  res.ok = S.ib[4] >= 0;
  res.result = S.ib[4];
  res.Z = Z;
  res.key_lo_k = 0u;
  res.key_lo = key_lo;
  res.kdraw = kdraw;
  return res;
}

// ------------------------------------------------ dense top-p rows
// Top-p threshold of a row without top-k whose nucleus the candidates do not
// hold (it reaches below their floor), by two re-streams:
//   1. the masses of the row's entries by high key byte (lane-private
//      fixed-point sums, as the radix path's first pass) give the byte bin hb
//      where the running mass from the top reaches p S;
//   2. per (round, warp) segment, the masses of the entries above bin hb,
//      and every entry of bin hb and the 32 keys below it (room for tie
//      floors) -- the bracket [lo, hi] -- (key, index) in the candidate
//      regions.
// The bracket's exact per-key counts then give tau_p (the first key, from
// hi down, where the mass above hi plus the bracket's mass from hi down
// reaches p S), and each segment's nucleus mass (its mass above hi plus its
// bracket entries at or above tau_p, in index order) is left in S.ss / S.sq
// (reference M) for the segment draw, which needs no further pass.  Returns
// false, with nothing decided, when a warp's region overflows or the
// crossing falls outside the bracket (the fixed-point bin sums can place it
// one bin off); the caller then takes the radix path.
template <int DT>
__device__ bool dense_topp(const KParams& P, RSmem& S, int row, int R, uint32_t kmax, float M, float T, float rT,
                           float pp, float S_all, uint32_t key_cut, int& ph, uint32_t* key_lo_out) {
  using C = Codec<DT, 16>;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float target = __fmul_rn(pp, S_all);
  lp_zero(S);
  stream_row<DT>(P, S, row, 0, R, [&](int, const uint4*, uint32_t (&raw)[8], uint32_t (&w)[8], int nv) {
    float e[kEPT];
    masses16<DT>(raw, T, rT, M, e);
#pragma unroll
    for (int j = 0; j < kEPT; ++j) {
      const uint32_t key = ECAH_RKEY(w, j);
      if (j < nv && key >= key_cut)
        atomicAdd(&S.lp[((key >> 8) << 5) | static_cast<uint32_t>(lane)], to_fixed(e[j], kFx));
    }
  });
  float* l0 = reinterpret_cast<float*>(&S.stage[0][0]);
  if (tid < 256) {
    unsigned long long acc = 0ull;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) acc += S.lp[(tid << 5) | ((j + tid) & 31)];
    l0[tid] = static_cast<float>(acc) * kFxInv;
  }
  __syncthreads();
  if (tid < 32) {
    int b;
    float ab;
    warp_select_seq<float, 256, true>(l0, target, &b, &ab);
    if (lane == 0) S.ib[2] = b;
  }
  __syncthreads();
  const uint32_t hb = static_cast<uint32_t>(S.ib[2]);
  if ((hb << 8) > kmax) return false;
  const uint32_t hi = min((hb << 8) | 255u, kmax);
  const uint32_t lo = ((hb << 8) >= 32u) ? (hb << 8) - 32u : 0u;

  // pass 2: masses above hi per segment, bracket entries into the regions
  int fill = 0;
  bool ovf = false;
  stream_row<DT>(P, S, row, 0, R, [&](int r, const uint4* st, uint32_t (&raw)[8], uint32_t (&w)[8], int nv) {
    float e[kEPT];
    masses16<DT>(raw, T, rT, M, e);
    float a = 0.f;
    uint32_t sb = 0u;
#pragma unroll
    for (int j = 0; j < kEPT; ++j) {
      const uint32_t key = ECAH_RKEY(w, j);
      if (j < nv) {
        if (key > hi) a += e[j];
        else if (key >= lo) sb |= 1u << j;
      }
    }
    a = warp_sum(a);
    if (lane == 0) { S.ss[r * kNW + warp] = a; S.sq[r * kNW + warp] = kRelM; }
    const int c = __popc(sb);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
    if (fill + total > kCBW) {
      ovf = true;
    } else if (!ovf) {
      const uint16_t* sr = reinterpret_cast<const uint16_t*>(st);
      int o = warp * kCBW + fill + incl - c;
      for (uint32_t m = sb; m; m &= m - 1u) {
        const int j = __ffs(m) - 1;
        S.ckey[o] = static_cast<uint16_t>(key16(sr[kEPT * lane + j]));
        S.cidx[o] = static_cast<uint32_t>(r * kRound + kEPT * tid + j);
        ++o;
      }
      fill += total;
    }
  });
  if (__syncthreads_or(ovf)) return false;
  unsigned* cnth = reinterpret_cast<unsigned*>(&S.stage[0][0]) + kCntOff;  // bin b = key hi - b
  for (int i = tid; i < kHB; i += kT) cnth[i] = 0u;
  fill = gather_candidates(S, fill, ph);
  for (int i = tid; i < fill; i += kT) atomicAdd(&cnth[hi - gkey(S)[i]], 1u);
  // mass above the bracket: the segments' sums
  const int nseg = R * kNW;
  const float A = rsum_f(tid < nseg ? S.ss[tid] : 0.f, S, ph);   // barrier inside: cnth complete
  float e4[4], se = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int b = tid * 4 + j;
    const unsigned cn = cnth[b];
    e4[j] = (cn && static_cast<uint32_t>(b) <= hi - lo) ? __fmul_rn(static_cast<float>(cn), mass_of(C::value(hi - static_cast<uint32_t>(b)), T, rT, M)) : 0.f;
    se += e4[j];
  }
  float btot;
  const float exb = rscan_f(se, S, ph, &btot);
  if (!(A < target) || !(A + btot >= target)) return false;   // the crossing lies outside the bracket
  int mine = INT_MAX;
  if (se > 0.f && A + exb + se >= target) {
    float run = A + exb;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (mine == INT_MAX && e4[j] > 0.f && run + e4[j] >= target) mine = tid * 4 + j;
      run += e4[j];
    }
    if (mine == INT_MAX) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (e4[j] > 0.f) mine = tid * 4 + j;
    }
  }
  unsigned bsel = rmin_u(static_cast<unsigned>(mine), S, ph);
  if (bsel == static_cast<unsigned>(INT_MAX)) {
    // reached only after rounding: the last non-zero bin
    int last = -1;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (e4[j] > 0.f) last = tid * 4 + j;
    bsel = static_cast<unsigned>(static_cast<int>(rmax_u(static_cast<unsigned>(last + 1), S, ph)) - 1);
    if (bsel == 0xFFFFFFFFu) return false;
  }
  const uint32_t key_lo = tie_floor<DT, 16>(hi - bsel, T);
  if (key_lo < lo) return false;
  // each segment's bracket entries at or above key_lo, in index order
  if (tid < nseg) {
    const int wi = (tid & 31) * 32 + (tid >> 5);   // gather_candidates: [warp][round] counts and offsets
    const unsigned b0 = S.lp[1024 + wi], n = S.lp[wi];
    float add = 0.f;
    for (unsigned i = b0; i < b0 + n; ++i) {
      const uint32_t key = gkey(S)[i];
      if (key >= key_lo) add += mass_of(C::value(key), T, rT, M);
    }
    S.ss[tid] += add;
  }
  __syncthreads();
  *key_lo_out = key_lo;
  return true;
}

// ------------------------------------------------ vocabulary-parallel local step
// Where row `row`'s list and count go: this rank's own buffers, or, in the
// fused step (FUSED), this rank's slot of exchange buffer h (every rank h,
// epoch parity `par`).
template <bool FUSED>
__device__ __forceinline__ unsigned long long* vp_list(const KParams& P, int row, int h, unsigned par) {
  if constexpr (!FUSED) return P.vp_cand + static_cast<long long>(row) * P.cand_cap;
  return reinterpret_cast<unsigned long long*>(static_cast<char*>(P.vp_base[h]) + P.vp_lcand) +
         ((static_cast<long long>(par) * P.vp_world + P.vp_rank) * P.vp_maxb + row) * P.cand_cap;
}
template <bool FUSED>
__device__ __forceinline__ int* vp_count_slot(const KParams& P, int row, int h, unsigned par) {
  if constexpr (!FUSED) return P.vp_count + row;
  return reinterpret_cast<int*>(static_cast<char*>(P.vp_base[h]) + P.vp_lcount) +
         (static_cast<long long>(par) * P.vp_world + P.vp_rank) * P.vp_maxb + row;
}
template <bool FUSED>
__device__ __forceinline__ void vp_put(const KParams& P, int row, unsigned par, int o, unsigned long long v) {
  if (o >= P.cand_cap) return;
  const int nd = FUSED ? P.vp_world : 1;
  for (int h = 0; h < nd; ++h) vp_list<FUSED>(P, row, h, par)[o] = v;
}
template <bool FUSED>
__device__ __forceinline__ void vp_put_count(const KParams& P, int row, unsigned par, int c) {
  const int nd = FUSED ? P.vp_world : 1;
  for (int h = 0; h < nd; ++h) *vp_count_slot<FUSED>(P, row, h, par) = c;
}

// After the stream of a slice (P.V entries, first global id P.vocab_offset):
// the slice's k-th largest key kth -- exact, from the per-key counts of the
// candidates, which hold every entry with key >= F, or by radix select when
// kth lies below F -- and every entry with key >= kth (ties included) in
// vocab order as (key << 32 | global id): the first cand_cap of them, and
// their count.
template <int DT, bool FUSED>
__device__ void vp_emit(const KParams& P, RSmem& S, int row, int R, int k, uint32_t kmax, uint32_t F, int fill,
                        bool cand, int& ph, unsigned par) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned gofs = static_cast<unsigned>(P.vocab_offset);
  if (cand) {
    unsigned* cnth = reinterpret_cast<unsigned*>(&S.stage[0][0]) + kCntOff;   // zeroed before the gather
    if (kmax >= static_cast<uint32_t>(kHB) && F < kmax - static_cast<uint32_t>(kHB - 1))
      F = kmax - static_cast<uint32_t>(kHB - 1);
    for (int i = tid; i < fill; i += kT) {
      const unsigned key = gkey(S)[i];
      if (key >= F) atomicAdd(&cnth[kmax - key], 1u);
    }
    __syncthreads();
    int tot;
    const unsigned b = cnth_select(cnth, k, S, ph, &tot);
    if (b != static_cast<unsigned>(INT_MAX) && kmax - b >= F) {
      const uint32_t kth = kmax - b;
      // the candidates in vocab order: 8 consecutive per thread
      const int b0 = tid * 8;
      unsigned m8 = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (b0 + j < fill && gkey(S)[b0 + j] >= kth) m8 |= 1u << j;
      int total;
      int o = rscan_i(__popc(m8), S, ph, &total);
      for (; m8; m8 &= m8 - 1u) {
        const int i = b0 + __ffs(m8) - 1;
        vp_put<FUSED>(P, row, par, o, (static_cast<unsigned long long>(gkey(S)[i]) << 32) | (gofs + gidx(S)[i]));
        ++o;
      }
      if (tid == 0) vp_put_count<FUSED>(P, row, par, total);
      return;
    }
  }
  // kth below the candidates: radix select, then per (round, warp) segment
  // the count of entries >= kth, their offsets, and the entries
  const uint32_t kth = radix_kth<DT>(P, S, row, R, static_cast<unsigned>(k));
  int* segc = reinterpret_cast<int*>(S.ss);
  stream_row<DT>(P, S, row, 0, R, [&](int r, const uint4*, uint32_t (&)[8], uint32_t (&w)[8], int nv) {
    int c = 0;
#pragma unroll
    for (int j = 0; j < kEPT; ++j) c += (j < nv && ECAH_RKEY(w, j) >= kth) ? 1 : 0;
    c = __reduce_add_sync(0xFFFFFFFFu, c);
    if (lane == 0) segc[r * kNW + warp] = c;
  });
  int total;
  const int off = rscan_i(tid < R * kNW ? segc[tid] : 0, S, ph, &total);
  if (tid < R * kNW) segc[tid] = off;
  stream_row<DT>(P, S, row, 0, R, [&](int r, const uint4*, uint32_t (&)[8], uint32_t (&w)[8], int nv) {
    unsigned m = 0u;
#pragma unroll
    for (int j = 0; j < kEPT; ++j)
      if (j < nv && ECAH_RKEY(w, j) >= kth) m |= 1u << j;
    const int c = __popc(m);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    int o = segc[r * kNW + warp] + incl - c;
    const unsigned e0 = gofs + static_cast<unsigned>(r * kRound + kEPT * tid);
#pragma unroll
    for (int j = 0; j < kEPT; ++j) {
      if ((m >> j) & 1u) {
        vp_put<FUSED>(P, row, par, o, (static_cast<unsigned long long>(ECAH_RKEY(w, j)) << 32) | (e0 + j));
        ++o;
      }
    }
  });
  if (tid == 0) vp_put_count<FUSED>(P, row, par, total);
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Fused step, once the lists and counts of all this CTA's rows are stored
// into every rank's buffer: after a CTA barrier one thread per rank fences
// at system scope (one fence for all the rows) and sets the rows' flags in
// that rank's buffer (release, system scope).
__device__ __forceinline__ void vp_signal(const KParams& P, unsigned epoch) {
  __syncthreads();
  if (static_cast<int>(threadIdx.x) < P.vp_world) {
    __threadfence_system();
    unsigned* fl = reinterpret_cast<unsigned*>(static_cast<char*>(P.vp_base[threadIdx.x]) + P.vp_lflag) +
                   static_cast<long long>(P.vp_rank) * P.vp_maxb;
    for (int row = blockIdx.x; row < P.B; row += gridDim.x) st_release_sys(fl + row, epoch);
  }
}

// The fused step's wait (bounded) for every rank's list of a row, then the
// merge and the draw, by merge group g of kMergeT threads: the CTA merges
// kMergeGroups rows at a time.  Defined with the merge (vp_kernel.cuh).
constexpr int kMergeT = 256;
constexpr int kMergeGroups = kT / kMergeT;
template <int DT>
__device__ __noinline__ void vp_fused_finish(const KParams& P, RSmem& S, int row, unsigned epoch, int g);

// ------------------------------------------------------------ the kernel
// One body for the sampler (VPM 0), the vocabulary-parallel local step (VPM
// 1: candidates only, then vp_emit) and the fused vocabulary-parallel step
// (VPM 2: vp_emit into every rank's exchange buffer, then vp_fused_finish).
template <int DT, bool SPLIT, int VPM>
__device__ __forceinline__ void row_body(const KParams& P) {
  constexpr bool VPL = VPM != 0, FUSED = VPM == 2;
  using C = Codec<DT, 16>;
  extern __shared__ __align__(16) unsigned char dsm[];
  RSmem& S = *reinterpret_cast<RSmem*>(dsm);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = (P.V + kRound - 1) / kRound;
  const int PP = SPLIT ? P.parts : 1;   // CTAs per row: each streams a run of rounds
  // fused step: this step's epoch (every row reads it before the last row
  // to finish advances it) and its exchange parity
  unsigned epoch = 0u;
  if constexpr (FUSED) epoch = *static_cast<volatile unsigned*>(P.vp_base[P.vp_rank]) + 1u;
  const unsigned par = epoch & 1u;

  for (int unit = blockIdx.x; unit < P.B * PP; unit += gridDim.x) {
    const int row = unit / PP, part = unit - row * PP;
    const int r0 = (R * part) / PP, r1 = (R * (part + 1)) / PP;
    int ph = 0;
    const float T = P.temperature[row];
    const int kk = P.top_k[row];
    const int k_eff = (kk <= 0 || kk >= P.V) ? P.V : kk;
    const float pp = P.top_p[row];
    const bool topk = k_eff < P.V;
    const bool topp = (pp > 0.f && pp < 1.f);
    const bool sampled = T > 0.f;
    const bool t1 = (T == 1.0f);
    const float rT = __frcp_rn(T);
    int N = !sampled ? 0 : (topk ? (k_eff <= kMaxN ? k_eff : 0) : (topp ? kDenseN : 0));
    if constexpr (VPL) {
      // k = top_k, the whole vocabulary when off, 1 for greedy rows; rows
      // whose list cannot hold k entries get count k and no list (the merge
      // refuses them)
      const long long kr = !sampled ? 1 : ((kk <= 0 || kk >= P.vocab_total) ? P.vocab_total : kk);
      N = static_cast<int>(min(kr, static_cast<long long>(P.V)));
      if (N > P.cand_cap) {
        if (tid == 0) vp_put_count<FUSED>(P, row, par, N);
        __syncthreads();
        continue;
      }
    }
    const bool mass_all = !VPL && sampled && !topk;   // S over the whole row
    const bool segs = mass_all && !topp;              // draw from segment sums
    // unsplit top-k rows record chunk top keys instead of keeping
    // candidates (lean_finish)
    const bool lean = !SPLIT && !VPL && N > 0 && topk && R <= kRecRounds;
    // unsplit top-p rows without top-k record each chunk's two largest keys
    // (plean_finish)
    const bool plean = !SPLIT && !VPL && mass_all && topp && R <= kRec2Rounds;
    if (plean) N = 0;

    // running state
    unsigned best = 0u;       // thread max key
    int bround = r0;          // first round where this thread met it
    unsigned f = 0u;          // candidate floor
    int fill = 0;
    bool overflow = (N == 0);

    // the row's uniform (or the Philox state) lands in shared memory with
    // thread 0's first stream copies, so it is there when the row finishes
    // (the vocabulary-parallel steps draw elsewhere and may pass neither)
    if (!VPL && tid == 0 && sampled) {
      if (P.uniforms) {
        cp_async4(&S.upre, P.uniforms + row);
      } else if (P.philox_state) {
        cp_async8(&S.pre[0], P.philox_state);
        cp_async8(&S.pre[1], P.philox_state + 1);
      }
    }
    if (row_has_penalty(P, row)) bucket_penalties<DT>(P, S, row, ph);
    uint32_t hwhi = 0u;       // record rows: top of the records' histogram
    if (plean)
      for (int i = tid; i < kPleanNB; i += kT) S.lp[i] = 0u;   // the stream's first barrier orders it
    uint32_t kcut = 0u;       // mass rows: warps whose keys all lie below skip their masses
    const uint32_t kinf = C::from_val(INFINITY), kninf = C::from_val(-INFINITY);

    // The round body, specialised per row mode at compile time (bit 0:
    // masses over the whole row; bit 1: per-segment masses; bit 2:
    // candidates), so each mode's stream loop carries only its own work.
    auto round_body = [&](auto mode, int r, const uint4* st, uint32_t (&raw)[8], uint32_t (&w)[8], int nv) {
      constexpr int MD = decltype(mode)::value;
      // bit 1: segment masses (the same code); bit 3: top-key records; bit 4: top-two records
      constexpr bool kMass = (MD & 1) != 0, kCand = (MD & 4) != 0, kRec = (MD & 8) != 0, kRec2 = (MD & 16) != 0;
      uint32_t tm;   // padding keys are 0
      if constexpr (kRec2) {
        const uint32_t t12 = top2_16(w);
        recs2(S)[(r - r0) * kT + tid] = t12;
        tm = t12 & 0xFFFFu;
        if (r != r0) plean_count(S, t12, hwhi);   // round r0's wait for the window
      } else {
        const uint32_t m2 = max16x2(max16x2(max16x2(w[0], w[1]), max16x2(w[2], w[3])),
                                    max16x2(max16x2(w[4], w[5]), max16x2(w[6], w[7])));
        tm = max(m2 & 0xFFFFu, m2 >> 16);
      }
      if constexpr (kRec) recs(S)[(r - r0) * kT + tid] = static_cast<uint16_t>(tm);
      if (tm > best) { best = tm; bround = r; }
      uint32_t k0 = 0u;  // max of the part's first round (that round only)
      if ((kMass || kCand) && r == r0 && (mass_all || !overflow)) k0 = rmax_u(tm, S, ph);

      if constexpr (kMass) {
        if (r == r0) {
          // entries with y below y0 - 36 T have mass below e^-36 relative to
          // the row max; all of them together stay below V e^-36 < 1e-9 of S
          const float ylo = __fsub_rn(C::value(k0), __fmul_rn(36.0f, T));
          kcut = (ylo > -INFINITY) ? C::from_val(ylo) : 0u;
        }
        // Segment (round, warp) masses 2^(z log2e - c) against the segment's
        // own reference c = z_max log2e, so no mass overflows whatever M
        // turns out to be.  Full rounds skip the NaN guard: a NaN logit makes
        // its segment sum NaN, which sends the row to the exact fallback.
        float rs = 0.f, cq = -INFINITY;
        if (__any_sync(0xFFFFFFFFu, tm >= kcut)) {
          uint32_t tr = tm;
          if (tm > kinf) {
            // NaN keys lie above +inf: the reference is the max of the others
            tr = 0u;
#pragma unroll
            for (int j = 0; j < kEPT; ++j) {
              const uint32_t key = ECAH_RKEY(w, j);
              if (key <= kinf) tr = max(tr, key);
            }
          }
          const uint32_t kw = __reduce_max_sync(0xFFFFFFFFu, tr);
          if (kw > kninf) {
            const float yw = C::value(kw);
            cq = __fmul_rn(t1 ? yw : __fdiv_rn(yw, T), kLog2e);
            if (t1) rs = (r < R - 1) ? seg_masses<DT, true, false>(raw, T, rT, cq) : seg_masses<DT, true, true>(raw, T, rT, cq);
            else rs = (r < R - 1) ? seg_masses<DT, false, false>(raw, T, rT, cq) : seg_masses<DT, false, true>(raw, T, rT, cq);
          }
        }
        const float ws = warp_sum(rs);
        if (lane == 0) { S.ss[r * kNW + warp] = ws; S.sq[r * kNW + warp] = cq; }
      }
      if constexpr (kRec2) {
        if (r == r0) {
          // the records' histogram covers keys up to round 0's max plus kPleanHead
          hwhi = min(k0 + static_cast<uint32_t>(kPleanHead), 0xFFFFu);
          plean_count(S, recs2(S)[tid], hwhi);
        }
      }

      if constexpr (kCand) {
      if (!overflow) {
        if (r == r0) {
          // First floor: the N0-th largest of the threads' round-0 maxima,
          // from counts of the 4096 keys below the round's max k0 in 256 bins
          // of 16 (the lowest key of the bin where N0 is reached).  N0
          // threads hold a key at or above it, so the round's N0-th largest
          // key is never below it.  Top-k rows take N0 = k (the row's k-th
          // largest key is never below it either); top-p rows scale N to the
          // round's share of the row, so about N entries pass in all.
          const int n0 = round_len(P.V, r0);
          const int N0 = (VPL || topk) ? N : max(1, static_cast<int>((static_cast<long long>(N) * n0 + P.V - 1) / P.V));
          if (tid < 256) S.h256[tid] = 0u;
          __syncthreads();
          const uint32_t d0 = k0 - tm;
          if (nv > 0 && d0 < 4096u) atomicAdd(&S.h256[d0 >> 4], 1u);
          __syncthreads();
          unsigned above;
          const int b = h256_select_asc(S, static_cast<unsigned>(N0), &above);
          const uint32_t d = (b >= 0) ? static_cast<uint32_t>(b) * 16u + 15u : 4095u;
          f = (k0 > d) ? max(k0 - d, 1u) : 1u;  // key 0 is padding
        }
        // survivor bits (key >= f >= 1; padding keys are 0 and never
        // survive): bit q = entry 2q, bit 16 + q = entry 2q + 1
        auto survivors = [&](unsigned fl) -> uint32_t {
          if (!__any_sync(0xFFFFFFFFu, tm >= fl)) return 0u;
          const uint32_t fm2 = (fl - 1u) * 0x00010001u;
          uint32_t sb = 0u;
#pragma unroll
          for (int q = 0; q < 8; ++q) sb |= surv2(w[q], fm2) << q;
          return sb;
        };
        // warp-level exclusive prefix of the lanes' survivor counts: one
        // ballot when no lane holds more than one, else a shuffle scan
        auto lane_scan = [&](uint32_t bits, int* tot) -> int {
          const int c = __popc(bits);
          const unsigned nz = __ballot_sync(0xFFFFFFFFu, c != 0);
          if (!__any_sync(0xFFFFFFFFu, c > 1)) {
            *tot = __popc(nz);
            return __popc(nz & ((1u << lane) - 1u));
          }
          int incl = c;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += y;
          }
          *tot = __shfl_sync(0xFFFFFFFFu, incl, 31);
          return incl - c;
        };
        uint32_t sb = survivors(f);
        int total;
        int off = lane_scan(sb, &total);
        if (fill + total > kCBW) {
          // raise the warp's floor toward the kKeepW-th largest key of its
          // region and this round's survivors, drop what falls below
          const unsigned nf = wcand_nth(S, fill, w, nv, f, __reduce_max_sync(0xFFFFFFFFu, best),
                                        static_cast<unsigned>(min(N, kKeepW)));
          if (nf > f) {
            f = nf;
            fill = wcand_compact(S, fill, f);
          }
          sb = survivors(f);
          off = lane_scan(sb, &total);
          if (fill + total > kCBW) overflow = true;
        }
        if (!overflow) {
          // append in vocab order: a survivor's slot is the lane's offset
          // plus the survivors among its lower entries; its key is re-read
          // from the stage
          const uint16_t* sr = reinterpret_cast<const uint16_t*>(st);
          const uint32_t base = static_cast<uint32_t>(r * kRound + kEPT * tid);
          const int o = warp * kCBW + fill + off;
          uint32_t m = sb;
          while (m) {
            const int bit = __ffs(m) - 1;
            m &= m - 1u;
            const int q = bit & 15, h = bit >> 4;
            const int e = 2 * q + h;
            const uint32_t lower = (((1u << q) - 1u) * 0x00010001u) | (static_cast<uint32_t>(h) << q);
            const int pos = o + __popc(sb & lower);
            S.ckey[pos] = static_cast<uint16_t>(key16(sr[kEPT * lane + e]));
            S.cidx[pos] = base + static_cast<uint32_t>(e);
          }
          fill += total;
        }
      }
      }
    };
    using std::integral_constant;
    const int smode = lean ? 8 : (plean ? 17 : ((mass_all ? 1 : 0) | (segs ? 2 : 0) | (!overflow ? 4 : 0)));
#define ECAH_ROUND(M) stream_row<DT>(P, S, row, r0, r1, [&](int r, const uint4* st, uint32_t (&raw)[8], uint32_t (&w)[8], int nv) { round_body(integral_constant<int, M>{}, r, st, raw, w, nv); })
    switch (smode) {
      case 0: ECAH_ROUND(0); break;
      case 1: ECAH_ROUND(1); break;
      case 3: ECAH_ROUND(3); break;
      case 4: ECAH_ROUND(4); break;
      case 5: ECAH_ROUND(5); break;
      case 8: ECAH_ROUND(8); break;
      case 17: ECAH_ROUND(17); break;
      default: ECAH_ROUND(7); break;   // no row mode sets other bits together
    }
#undef ECAH_ROUND

    unsigned* cnth = reinterpret_cast<unsigned*>(&S.stage[0][0]) + kCntOff;  // [kHB] counts, bin b = key kmax - b
    if (N > 0 && !lean) {
      // the warps' floors and regions -> one floor F (their max) and one
      // buffer in vocab order holding every entry of the row with key >= F
      overflow = __syncthreads_or(overflow) != 0;
      if (!overflow) {
        for (int i = tid; i < kHB; i += kT) cnth[i] = 0u;   // outside the gather's scratch
        fill = gather_candidates(S, fill, ph);
      }
    }
    bool cand = N > 0 && !overflow && !lean;   // every entry with key >= f is in the buffer

    // ------------------------------------------------ row max and greedy
    unsigned kmax, fmax;
    rmax2_u(best, N > 0 ? f : 0u, S, ph, &kmax, &fmax);
    if constexpr (VPL) {
      vp_emit<DT, FUSED>(P, S, row, R, N, kmax, fmax, fill, cand, ph, par);
      __syncthreads();  // shared state is reused by the next row
      continue;
    }
    if (N > 0) f = fmax;
    // The lowest index of the max: greedy rows and split rows need it now;
    // sampled rows only when no entry has finite mass (see `none`), so they
    // scan the candidates while the buffer is intact and reduce later.
    unsigned firstc = 0xFFFFFFFFu;
    auto scan_first = [&]() {
      if (cand) {
        // the max is at or above every floor: all its entries are candidates
        for (int i = tid; i < fill; i += kT)
          if (gkey(S)[i] == kmax) firstc = min(firstc, gidx(S)[i]);
      } else if (best == kmax) {
        // the lowest index of kmax among this thread's entries of round bround
        // (fetching them for every thread ahead of the barrier measured slower)
        const int e0 = bround * kRound + kEPT * tid;
        float yv[kEPT];
        load16<DT>(P, S, row, e0, yv);
#pragma unroll
        for (int j = 0; j < kEPT; ++j)
          if (firstc == 0xFFFFFFFFu && e0 + j < P.V && C::from_val(yv[j]) == kmax) firstc = static_cast<unsigned>(e0 + j);
      }
    };
    const bool greedy_now = !(T > 0.f) || !isfinite(__fdiv_rn(C::value(kmax), T));
    unsigned first = 0xFFFFFFFFu;
    if (SPLIT || greedy_now) {
      scan_first();
      first = rmin_u(firstc, S, ph);
    } else if (cand) {
      scan_first();
    }

    if constexpr (SPLIT) {
      PartState m{kmax, first, f, fill, overflow, cand};
      if (!part_exchange(P, S, row, part, PP, r0, r1, R, N, mass_all, ph, m)) continue;   // another part finishes
      kmax = m.kmax; first = m.first; f = m.f; fill = m.fill; overflow = m.overflow; cand = m.cand;
    }
    const float ymax = C::value(kmax);
    const float M = __fdiv_rn(ymax, T);
    const bool greedy = !(T > 0.f) || !isfinite(M);
    int result = static_cast<int>(first == 0xFFFFFFFFu ? 0u : first);
    RowFin* fin = static_cast<RowFin*>(P.ws_fin) + row;
    const float u = greedy ? 0.f : (P.uniforms ? S.upre : row_uniform(S.pre[0], S.pre[1], static_cast<uint64_t>(row)));

    if (greedy) {
      if (tid == 0) {
        if (P.row_stats) {
          float* st = P.row_stats + 4ll * row;
          st[0] = ymax; st[1] = ymax; st[2] = ymax; st[3] = 1.0f;
        }
        fin->M = ymax; fin->Z = 1.0f; fin->kdraw = 0u; fin->mode = 1; fin->idx = result;
      }
    } else {
      const uint32_t key_cut = zero_mass_cut<DT, 16>(M, T);
      // whole-row mass rescaled to M
      // segment masses were taken relative to references <= M: this
      // thread's share of the whole-row mass, summed behind the next barrier
      float S_all = 0.f;
      if (mass_all) {
        const float sm = warp_sum(seg_mass(S, tid, R * kNW, M));
        if (lane == 0) S.part[warp] = sm;
      }
      uint32_t key_lo_k = 0u, key_lo = 0u;
      uint32_t F = f;
      const bool thr = cand && (topk || topp);
      if (thr) {
        if (kmax >= static_cast<uint32_t>(kHB) && F < kmax - static_cast<uint32_t>(kHB - 1))
          F = kmax - static_cast<uint32_t>(kHB - 1);   // entries below stay out of the histogram
        for (int i = tid; i < fill; i += kT) {
          const unsigned key = gkey(S)[i];
          if (key >= F) atomicAdd(&cnth[kmax - key], 1u);
        }
      }
      __syncthreads();
      bool mass_ok = true;
      if (mass_all) {
        S_all = warp_sum(S.part[lane]);
        mass_ok = isfinite(S_all);
      }
      bool fast = (!overflow || segs) && mass_ok;
      // record rows: floor, thresholds and draw from the chunk records; when
      // they decide nothing, the re-streaming paths below take the row
      bool lean_done = false;
      float lean_Z = 0.f;
      int lean_result = 0;
      if (lean) {
        const LeanRes lr = lean_finish<DT>(P, S, row, R, kmax, M, T, rT, k_eff, topp, pp, key_cut, u, ph);
        if (lr.ok) {
          lean_done = true;
          key_lo_k = lr.key_lo_k;
          key_lo = lr.key_lo;
          lean_Z = lr.Z;
          lean_result = lr.result;
        } else {
          fast = false;   // the re-streaming paths below
        }
      }
      if (plean && mass_ok) {
        const LeanRes lr = plean_finish<DT>(P, S, row, R, kmax, M, T, rT, pp, S_all, key_cut, u, hwhi, ph);
        if (lr.ok) {
          lean_done = true;
          fast = true;
          key_lo = lr.key_lo;
          lean_Z = lr.Z;
          lean_result = lr.result;
        }
      }
      if (thr) {
        const int Bmax = static_cast<int>(kmax - F);
        // top-k: the k-th largest key among the candidates
        if (topk) {
          int tot;
          const unsigned bsel = cnth_select(cnth, k_eff, S, ph, &tot);
          if (tot < k_eff || bsel == static_cast<unsigned>(INT_MAX)) {
            fast = false;
          } else {
            key_lo_k = tie_floor<DT, 16>(kmax - bsel, T);   // every thread, same value
            if (key_lo_k < F) fast = false;
          }
        }
        key_lo = key_lo_k;
        if (fast && topp) {
          const int bk = topk ? static_cast<int>(kmax - key_lo_k) : Bmax;
          float m4[4];
          float s4 = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int b = tid * 4 + j;
            const unsigned cn = cnth[b];
            m4[j] = (b <= bk && cn) ? __fmul_rn(static_cast<float>(cn), mass_of(C::value(kmax - static_cast<uint32_t>(b)), T, rT, M)) : 0.f;
            s4 += m4[j];
          }
          float tot;
          const float ex = rscan_f(s4, S, ph, &tot);
          const float S_K = topk ? tot : S_all;
          const float target = __fmul_rn(pp, S_K);
          int mine = INT_MAX;
          if (s4 > 0.f && ex + s4 >= target) {
            float acc = ex;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (mine == INT_MAX && m4[j] > 0.f && acc + m4[j] >= target) mine = tid * 4 + j;
              acc += m4[j];
            }
            if (mine == INT_MAX) {
              // rounding left the target unreached inside this thread: its last non-zero bin
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (m4[j] > 0.f) mine = tid * 4 + j;
            }
          }
          unsigned bsel = rmin_u(static_cast<unsigned>(mine), S, ph);
          const bool reached = tot >= target;
          if (bsel == static_cast<unsigned>(INT_MAX) && reached) {
            // the running total reaches the target only after rounding: last non-zero bin
            int last = -1;
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (m4[j] > 0.f) last = tid * 4 + j;
            bsel = static_cast<unsigned>(static_cast<int>(rmax_u(static_cast<unsigned>(last + 1), S, ph)) - 1);
          }
          if (!reached || bsel == static_cast<unsigned>(INT_MAX) || bsel == 0xFFFFFFFFu) {
            fast = false;
          } else {
            key_lo = max(tie_floor<DT, 16>(kmax - bsel, T), key_lo_k);   // every thread, same value
            if (key_lo < F) fast = false;
          }
        }
      }

      // rows without top-k whose nucleus reaches below the candidates
      bool segs_ready = false;
      if (!fast && mass_all && topp && mass_ok) {
        uint32_t kl;
        if (dense_topp<DT>(P, S, row, R, kmax, M, T, rT, pp, S_all, key_cut, ph, &kl)) {
          key_lo_k = 0u;
          key_lo = kl;
          segs_ready = true;
        }
      }
      if (!fast && !segs_ready) {
        // ---------------------------------- fallback: radix select by re-streaming
        key_lo_k = 0u;
        if (topk) key_lo_k = tie_floor<DT, 16>(radix_kth<DT>(P, S, row, R, static_cast<unsigned>(k_eff)), T);
        key_lo = key_lo_k;
        if (topp) {
          const uint32_t klo = max(key_lo_k, key_cut);
          lp_zero(S);
          float sk = 0.f;
          stream_row<DT>(P, S, row, 0, R, [&](int, const uint4*, uint32_t (&)[8], uint32_t (&w)[8], int nv) {
#pragma unroll
            for (int j = 0; j < kEPT; ++j) {
              const uint32_t key = ECAH_RKEY(w, j);
              if (j < nv && key >= klo) {
                const float e = mass_of(C::value(key), T, rT, M);
                sk += e;
                atomicAdd(&S.lp[((key >> 8) << 5) | static_cast<uint32_t>(lane)], to_fixed(e, kFx));
              }
            }
          });
          const float S_K = rsum_f(sk, S, ph);
          __syncthreads();
          float* l0 = reinterpret_cast<float*>(S.stage);
          if (tid < 256) {
            unsigned long long acc = 0ull;
#pragma unroll 8
            for (int j = 0; j < 32; ++j) acc += S.lp[(tid << 5) | ((j + tid) & 31)];
            l0[tid] = static_cast<float>(acc) * kFxInv;
          }
          __syncthreads();
          const float target = __fmul_rn(pp, S_K);
          if (tid < 32) {
            int b; float ab;
            warp_select_seq<float, 256, true>(l0, target, &b, &ab);
            if (lane == 0) S.ib[2] = b;
          }
          __syncthreads();
          const int hb = S.ib[2];
          lp_zero(S);
          float above = 0.f;
          stream_row<DT>(P, S, row, 0, R, [&](int, const uint4*, uint32_t (&)[8], uint32_t (&w)[8], int nv) {
#pragma unroll
            for (int j = 0; j < kEPT; ++j) {
              const uint32_t key = ECAH_RKEY(w, j);
              if (j < nv && key >= klo) {
                const int kb = static_cast<int>(key >> 8);
                if (kb == hb) atomicAdd(&S.lp[((key & 255u) << 5) | static_cast<uint32_t>(lane)], 1u);
                else if (kb > hb) above += mass_of(C::value(key), T, rT, M);
              }
            }
          });
          const float above_b = rsum_f(above, S, ph);
          lp_reduce(S);
          float* m1 = reinterpret_cast<float*>(S.stage);
          if (tid < 256) {
            const uint32_t key = (static_cast<uint32_t>(hb) << 8) | static_cast<uint32_t>(tid);
            const unsigned cn = S.h256[tid];
            m1[tid] = cn ? __fmul_rn(static_cast<float>(cn), mass_of(C::value(key), T, rT, M)) : 0.f;
          }
          __syncthreads();
          if (tid < 32) {
            int d; float ab;
            warp_select_seq<float, 256, true>(m1, __fsub_rn(target, above_b), &d, &ab);
            if (lane == 0) S.ib[3] = static_cast<int>(max(tie_floor<DT, 16>((static_cast<uint32_t>(hb) << 8) | static_cast<uint32_t>(d), T), key_lo_k));
          }
          __syncthreads();
          key_lo = static_cast<uint32_t>(S.ib[3]);
        }
      }

      const uint32_t kdraw = max(key_lo, key_cut);
      float Z = 0.f;
      bool none = false;
      if (lean_done) {
        Z = lean_Z;
        result = lean_result;
      } else if (fast && (topk || topp)) {
        // inverse CDF over the candidates, in vocab order (entries 8*tid .. 8*tid+7)
        float e[8];
        float s8 = 0.f;
        const int b0 = tid * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = b0 + j;
          e[j] = 0.f;
          if (i < fill) {
            const uint32_t key = gkey(S)[i];
            if (key >= kdraw) e[j] = mass_of(C::value(key), T, rT, M);
          }
          s8 += e[j];
        }
        const float ex = rscan_f(s8, S, ph, &Z);
        const float target = __fmul_rn(u, Z);
        int mine = INT_MAX, last = -1;
        float acc = ex;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (e[j] > 0.f) {
            last = b0 + j;
            if (mine == INT_MAX && acc + e[j] > target) mine = b0 + j;
            acc += e[j];
          }
        }
        unsigned pick, lastp;
        rminmax_u(static_cast<unsigned>(mine), static_cast<unsigned>(last + 1), S, ph, &pick, &lastp);
        if (pick != static_cast<unsigned>(INT_MAX)) result = static_cast<int>(gidx(S)[pick]);
        else if (lastp > 0u) result = static_cast<int>(gidx(S)[lastp - 1u]);
        else none = true;
      } else {
        // segment sums: from the stream (whole distribution) or a re-stream
        const int nseg = R * kNW;
        if (!(fast && segs) && !segs_ready) {
          stream_row<DT>(P, S, row, 0, R, [&](int r, const uint4*, uint32_t (&)[8], uint32_t (&w)[8], int nv) {
            float a = 0.f;
#pragma unroll
            for (int j = 0; j < kEPT; ++j) {
              const uint32_t key = ECAH_RKEY(w, j);
              if (j < nv && key >= kdraw) a += mass_of(C::value(key), T, rT, M);
            }
            a = warp_sum(a);
            if (lane == 0) { S.ss[r * kNW + warp] = a; S.sq[r * kNW + warp] = kRelM; }
          });
        }
        // per-segment mass relative to M, then the segment holding u * Z
        const float v = seg_mass(S, tid, nseg, M);
        const float ex = rscan_f(v, S, ph, &Z);
        const float target = __fmul_rn(u, Z);
        const int mine = (tid < nseg && v > 0.f && ex + v > target) ? tid : INT_MAX;
        unsigned pick, lastp;
        rminmax_u(static_cast<unsigned>(mine), static_cast<unsigned>(v > 0.f ? tid + 1 : 0), S, ph, &pick, &lastp);
        int seg;
        bool take_last = false;
        if (pick != static_cast<unsigned>(INT_MAX)) seg = static_cast<int>(pick);
        else if (lastp > 0u) { seg = static_cast<int>(lastp) - 1; take_last = true; }
        else { seg = -1; none = true; }
        if (seg >= 0) {
          // remaining target inside the segment (threads see the same prefix value)
          if (tid == seg) S.fb[0] = __fsub_rn(target, ex);
          __syncthreads();
          const float rem = S.fb[0];
          // re-load the segment's 512 entries: warp 0, 16 per lane
          if (warp == 0) {
            const int r = seg / kNW, sw = seg % kNW;
            const int e0 = r * kRound + sw * 512 + lane * kEPT;
            float ev[kEPT];
            float ls = 0.f;
            int lastj = -1;
            float yv[kEPT];
            load16<DT>(P, S, row, e0, yv);
#pragma unroll
            for (int j = 0; j < kEPT; ++j) {
              const int i = e0 + j;
              ev[j] = 0.f;
              if (i < P.V) {
                const uint32_t key = C::from_val(yv[j]);
                if (key >= kdraw) ev[j] = mass_of(yv[j], T, rT, M);
              }
              if (ev[j] > 0.f) lastj = j;
              ls += ev[j];
            }
            float incl = ls;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
              if (lane >= o) incl += y;
            }
            const float excl = incl - ls;
            const unsigned hit = take_last ? 0u : __ballot_sync(0xFFFFFFFFu, ls > 0.f && incl > rem);
            int L;
            bool last = take_last;
            if (hit) L = __ffs(hit) - 1;
            else {
              const unsigned nz = __ballot_sync(0xFFFFFFFFu, ls > 0.f);
              L = nz ? 31 - __clz(nz) : 0;
              last = true;
            }
            if (lane == L) {
              int pk = -1;
              float run = excl;
#pragma unroll
              for (int j = 0; j < kEPT; ++j) {
                if (pk < 0 && !last && ev[j] > 0.f) {
                  run += ev[j];
                  if (run > rem) pk = j;
                }
              }
              if (pk < 0) pk = max(lastj, 0);
              S.ib[4] = e0 + pk;
            }
          }
          __syncthreads();
          result = S.ib[4];
        }
      }
      if (none) {
        // no finite mass anywhere: the lowest index of the row max
        if constexpr (!SPLIT) {
          if (!cand) scan_first();   // from global memory: the stages may be gone
          first = rmin_u(firstc, S, ph);
        }
        result = static_cast<int>(first == 0xFFFFFFFFu ? 0u : first);
      }
      if (tid == 0) {
        if (P.row_stats) {
          float* st = P.row_stats + 4ll * row;
          st[0] = topk ? C::value(key_lo_k) : -INFINITY;
          st[1] = (topk || topp) ? C::value(key_lo) : -INFINITY;
          st[2] = M;
          st[3] = Z;
        }
        fin->M = M; fin->Z = Z; fin->kdraw = kdraw; fin->mode = none ? 2 : 0; fin->idx = result;
      }
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
    __syncthreads();  // shared state is reused by the next row
  }
  if constexpr (FUSED) {
    // every row of this CTA is out: flag them all, then wait for the other
    // ranks' lists of each and merge it (no CTA waits before it has flagged
    // all its own rows)
    vp_signal(P, epoch);
    const int g = tid / kMergeT;   // merge groups run independently from here on
    for (int i = g;; i += kMergeGroups) {
      const long long row = blockIdx.x + static_cast<long long>(i) * gridDim.x;
      if (row >= P.B) break;
      vp_fused_finish<DT>(P, S, static_cast<int>(row), epoch, g);
    }
  }
}

template <int DT, bool SPLIT>
__global__ void __launch_bounds__(kT, 1) row_sample_kernel(const __grid_constant__ KParams P) {
  row_body<DT, SPLIT, 0>(P);
}

// Vocabulary-parallel local step: per row of the slice, the entries at or
// above the slice's k-th largest key (vp_emit).  P.V is the slice length.
template <int DT>
__global__ void __launch_bounds__(kT, 1) vp_local_row_kernel(const __grid_constant__ KParams P) {
  row_body<DT, false, 1>(P);
}

#undef ECAH_RKEY

}  // namespace rk
}  // namespace ecah
