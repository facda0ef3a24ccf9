// Chunk staging and the probability kernel of the 16-bit samplers, plus the
// sequential warp select shared with the vocab-parallel kernels.
//
// stream_probs_kernel writes probs_out for rows the row kernel
// (row_kernel.cuh) finished: one CTA per (row, 8192-entry chunk), each
// re-reading its chunk once and writing mass / Z over the kept keys from the
// row's finished data (RowFin: M, Z, the lowest kept key, the mode).
#pragma once

#include "sampler_kernel.cuh"

namespace ecah {

constexpr int kSCH = 8192;                 // vocab entries per chunk
constexpr int kSVecs = kSCH / 8;           // 16-byte vectors per chunk
struct RowFin {    // what the probability kernel needs of a finished row
  float M, Z;
  unsigned kdraw;
  int mode;        // 0: mass / Z over keys >= kdraw; 1: one-hot at idx; 2: all zero
  int idx;
  int pad0, pad1, pad2;
};

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

// ----------------------------------------------------------- chunk staging
// Chunk c of `row` into `buf`: raw logits of the model dtype with the
// slot's penalties applied to its history tokens (penalise); entries
// past the row end read 0xFFFF (key 0, below every logit).
//
// issue_chunk starts the 16-byte cp.async copies of the whole vectors (no
// wait); complete_chunk, once they have landed, loads the ragged tail (and
// unaligned rows) with plain loads, pads, applies the penalty patch, and
// returns with the buffer complete.  Both are reached by the whole CTA.
__device__ __forceinline__ void issue_chunk(const KParams& P, uint4* buf, int row, int c, int n) {
  if (!P.vec_ok) return;
  const uint4* s4 = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(P.logits) +
                                                   logits_row_offset(P, row) + c * kSCH);
  const int nfull = n >> 3;
  for (int v = threadIdx.x; v < nfull; v += kThreads) cp_async16(buf + v, s4 + v);
}

template <int DT>
__device__ void complete_chunk(const KParams& P, uint4* buf, int row, int c, int n) {
  using Dt = DType<DT>;
  const int tid = threadIdx.x;
  const int c0 = c * kSCH;
  const uint16_t* src = static_cast<const uint16_t*>(P.logits) + logits_row_offset(P, row) + c0;
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
        raw[li] = static_cast<uint16_t>(Dt::to_raw(penalise<DT>(x, m, additive_term(P, row, cnt))));
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
__device__ __forceinline__ int chunk_len(const KParams& P, int c) { return min(kSCH, P.V - c * kSCH); }

// probs_out of the rows finished by the row kernel (launched after it)
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


}  // namespace ecah
