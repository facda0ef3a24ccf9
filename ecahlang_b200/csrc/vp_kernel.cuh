// Vocab-parallel sampling (fp16/bf16 logits): every rank holds a contiguous
// slice [vocab_offset, vocab_offset + vocab_local) of each row.
//
// vp_local_kernel (one CTA per row) keeps the slice in shared memory, applies
// the repetition-penalty patch of the row's history tokens that fall in the
// slice, finds the slice's k-th largest key (k = top_k, 1 for greedy rows)
// with a two-digit (8 | 8 bit) radix select, and writes every slice entry
// whose key is >= that key -- ties included -- in vocab order as
// (key << 32 | global id), up to cand_cap of them, plus their count.
//
// Because the row's k-th largest key is >= every slice's k-th largest key,
// the union of the slices' lists holds every entry of the row's top-k set.
// After an all-gather of the lists, vp_merge_kernel (one CTA per row, the
// same on every rank) takes the row max, the top-k threshold (exact counts
// per key of the merged entries), softmax masses, the top-p threshold and the
// inverse-CDF draw in global vocab order with the row's uniform, so every
// rank returns the same token.  Op order, masses and tie rules are those of
// the other sampler kernels.
#pragma once

#include "stream_kernel.cuh"

namespace ecah {
namespace vp {

constexpr int kLT = 512;                 // threads of the local kernel
constexpr int kLW = kLT / 32;
constexpr int kMaxLocal = 65536;         // slice entries held in shared memory
constexpr int kMT = 256;                 // threads of the merge kernel
constexpr int kMW = kMT / 32;
constexpr int kMaxMerged = 2048;         // world * cand_cap entries per row, at most
constexpr int kWin = 4096;               // merge histogram: keys below the row max

struct VParams {
  const void* logits;
  long long row_stride;
  int B, Vl, V, offset;
  const float* temperature;
  const int* top_k;
  const float* top_p;
  const float* rep_factor;
  const int* row_slot;
  const int* slot_len;
  const int* hist_tok;
  const int* hist_cnt;
  const float* hist_mval;
  int hist_cap, num_slots;
  int cap;                                // candidates per row and rank
  unsigned long long* cand;               // [B, cap] local lists
  int* count;                             // [B] local counts (> cap: truncated)
  int world;
  const unsigned long long* all_cand;     // [world, B, cap]
  const int* all_count;                   // [world, B]
  const float* uniforms;
  unsigned long long* philox_state;
  unsigned* done_counter;
  int* out;
  float* row_stats;
  int vec_ok;
};

// ------------------------------------------------------------ local step
struct LSmem {
  uint16_t raw[kMaxLocal];   // the slice (raw logits, penalised)
  unsigned lp[256 * 32];     // lane-private 256-bin histogram
  unsigned h[256];
  int wsum[kLW];
  int ib[4];
};

template <int DT>
__global__ void __launch_bounds__(kLT) vp_local_kernel(const __grid_constant__ VParams P) {
  using Dt = DType<DT>;
  extern __shared__ __align__(16) unsigned char dsm[];
  LSmem& S = *reinterpret_cast<LSmem*>(dsm);
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = P.Vl;
  const uint16_t* src = static_cast<const uint16_t*>(P.logits) + static_cast<long long>(row) * P.row_stride;

  // load the slice
  int done = 0;
  if (P.vec_ok) {
    const int nfull = n >> 3;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(S.raw);
    for (int v = tid; v < nfull; v += kLT) cp_async16(d4 + v, s4 + v);
    done = nfull << 3;
  }
  for (int i = done + tid; i < n; i += kLT) S.raw[i] = src[i];
  cp_async_wait_all();
  __syncthreads();
  if (P.row_slot) {
    const int slot = P.row_slot[row];
    if (slot >= 0 && slot < P.num_slots) {
      const int len = min(P.slot_len[slot], P.hist_cap);
      const float rf = P.rep_factor ? P.rep_factor[row] : 1.0f;
      const long long base = static_cast<long long>(slot) * P.hist_cap;
      for (int h = tid; h < len; h += kLT) {
        const int li = P.hist_tok[base + h] - P.offset;
        const int cnt = P.hist_cnt[base + h];
        if (cnt <= 0 || li < 0 || li >= n) continue;
        const float x = Dt::to_f32(S.raw[li]);
        const float m = P.hist_mval ? P.hist_mval[base + h] : penalty_divisor<DT>(cnt, rf);
        S.raw[li] = static_cast<uint16_t>(Dt::to_raw(Dt::round(__fdiv_rn(x, m))));
      }
    }
    __syncthreads();
  }

  const float T = P.temperature[row];
  const int kk = P.top_k[row];
  // rows without top-k keep every entry (they fit only in small slices)
  const long long k_row = (!(T > 0.f)) ? 1 : ((kk <= 0 || kk >= P.V) ? static_cast<long long>(P.V) : kk);
  const unsigned k = static_cast<unsigned>(min(k_row, static_cast<long long>(n)));

  // k-th largest key of the slice: high byte, then low byte
  for (int i = tid; i < 256 * 32; i += kLT) S.lp[i] = 0u;
  __syncthreads();
  for (int i = tid; i < n; i += kLT) atomicAdd(&S.lp[((key16(S.raw[i]) >> 8) << 5) | lane], 1u);
  __syncthreads();
  if (tid < 256) {
    unsigned acc = 0u;
    for (int j = 0; j < 32; ++j) acc += S.lp[(tid << 5) | ((j + tid) & 31)];
    S.h[tid] = acc;
  }
  __syncthreads();
  if (tid < 32) {
    int b; unsigned above;
    warp_select_seq<unsigned, 256, true>(S.h, k, &b, &above);
    if (lane == 0) { S.ib[0] = b; S.ib[1] = static_cast<int>(above); }
  }
  __syncthreads();
  const int hb = S.ib[0];
  const unsigned krem = k - static_cast<unsigned>(S.ib[1]);
  for (int i = tid; i < 256 * 32; i += kLT) S.lp[i] = 0u;
  __syncthreads();
  for (int i = tid; i < n; i += kLT) {
    const uint32_t key = key16(S.raw[i]);
    if (static_cast<int>(key >> 8) == hb) atomicAdd(&S.lp[((key & 255u) << 5) | lane], 1u);
  }
  __syncthreads();
  if (tid < 256) {
    unsigned acc = 0u;
    for (int j = 0; j < 32; ++j) acc += S.lp[(tid << 5) | ((j + tid) & 31)];
    S.h[tid] = acc;
  }
  __syncthreads();
  if (tid < 32) {
    int b; unsigned above;
    warp_select_seq<unsigned, 256, true>(S.h, krem, &b, &above);
    if (lane == 0) S.ib[2] = static_cast<int>((static_cast<uint32_t>(hb) << 8) | static_cast<uint32_t>(b));
  }
  __syncthreads();
  const uint32_t kth = static_cast<uint32_t>(S.ib[2]);

  // entries >= kth in vocab order: thread t owns a contiguous stretch
  const int per = (n + kLT - 1) / kLT;
  const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
  int cnt = 0;
  for (int i = i0; i < i1; ++i) cnt += (key16(S.raw[i]) >= kth) ? 1 : 0;
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) S.wsum[warp] = incl;
  __syncthreads();
  int base = 0, total = 0;
  for (int w = 0; w < kLW; ++w) {
    if (w < warp) base += S.wsum[w];
    total += S.wsum[w];
  }
  int o = base + incl - cnt;
  unsigned long long* dst = P.cand + static_cast<long long>(row) * P.cap;
  for (int i = i0; i < i1 && o < P.cap; ++i) {
    const uint32_t key = key16(S.raw[i]);
    if (key >= kth) {
      dst[o] = (static_cast<unsigned long long>(key) << 32) | static_cast<unsigned>(P.offset + i);
      ++o;
    }
  }
  if (tid == 0) P.count[row] = total;
}

// ------------------------------------------------------------ merge step
struct MSmem {
  unsigned long long c[kMaxMerged];   // merged entries, rank order (= vocab order)
  unsigned cnt[kWin];                 // counts per key, bin b = key kmax - b
  float red[kMW];
  unsigned ured[kMW];
  int ofs[65];
  int ib[8];
  float fb[8];
};

__device__ __forceinline__ unsigned mblock_max(unsigned v, unsigned* red) {
  v = __reduce_max_sync(0xFFFFFFFFu, v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned m = 0u;
  for (int w = 0; w < kMW; ++w) m = max(m, red[w]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ unsigned mblock_min(unsigned v, unsigned* red) {
  v = __reduce_min_sync(0xFFFFFFFFu, v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned m = 0xFFFFFFFFu;
  for (int w = 0; w < kMW; ++w) m = min(m, red[w]);
  __syncthreads();
  return m;
}

template <int DT>
__global__ void __launch_bounds__(kMT) vp_merge_kernel(const __grid_constant__ VParams P) {
  using C = Codec<DT, 16>;
  __shared__ MSmem S;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;

  // merged entries of the row: rank by rank (each rank's list is in vocab order)
  if (tid == 0) {
    int acc = 0, bad = 0;
    for (int g = 0; g < P.world; ++g) {
      const int c = P.all_count[static_cast<long long>(g) * P.B + row];
      if (c > P.cap) bad = 1;
      S.ofs[g] = acc;
      acc += min(c, P.cap);
    }
    S.ofs[P.world] = acc;
    S.ib[0] = bad;
  }
  __syncthreads();
  const int total = S.ofs[P.world];
  const bool truncated = S.ib[0] != 0;
  for (int g = 0; g < P.world; ++g) {
    const int c = S.ofs[g + 1] - S.ofs[g];
    const unsigned long long* src = P.all_cand + (static_cast<long long>(g) * P.B + row) * P.cap;
    for (int i = tid; i < c; i += kMT) S.c[S.ofs[g] + i] = src[i];
  }
  __syncthreads();

  const float T = P.temperature[row];
  const int kk = P.top_k[row];
  const int k_eff = (kk <= 0 || kk >= P.V) ? P.V : kk;
  const float pp = P.top_p[row];
  const bool topk = k_eff < P.V;
  const bool topp = (pp > 0.f && pp < 1.f);

  // row max and its lowest id
  unsigned km = 0u;
  for (int i = tid; i < total; i += kMT) km = max(km, static_cast<unsigned>(S.c[i] >> 32));
  const unsigned kmax = mblock_max(km, S.ured);
  unsigned fid = 0xFFFFFFFFu;
  for (int i = tid; i < total; i += kMT)
    if (static_cast<unsigned>(S.c[i] >> 32) == kmax) fid = min(fid, static_cast<unsigned>(S.c[i] & 0xFFFFFFFFu));
  const unsigned first = mblock_min(fid, S.ured);
  const float ymax = C::value(kmax);
  const float M = __fdiv_rn(ymax, T);
  const bool greedy = !(T > 0.f) || !isfinite(M);
  int result = static_cast<int>(first == 0xFFFFFFFFu ? 0u : first);
  float Z = 1.0f;
  uint32_t key_lo_k = kmax, key_lo = kmax;
  bool ok = total > 0 && !truncated;

  if (!greedy && ok) {
    float u;
    if (P.uniforms) u = P.uniforms[row];
    else u = row_uniform(__ldcg(&P.philox_state[0]), __ldcg(&P.philox_state[1]), static_cast<uint64_t>(row));
    const float rT = __frcp_rn(T);
    const uint32_t key_cut = zero_mass_cut<DT, 16>(M, T);
    // every entry with key >= F is in the merged list: F = the highest of the
    // ranks' k-th largest keys (the lowest key of each rank's list)
    unsigned fl = 0u;
    if (tid < P.world) {
      const int c = S.ofs[tid + 1] - S.ofs[tid];
      unsigned lo = 0xFFFFFFFFu;
      for (int i = 0; i < c; ++i) lo = min(lo, static_cast<unsigned>(S.c[S.ofs[tid] + i] >> 32));
      fl = (c > 0) ? lo : 0u;
    }
    uint32_t F = mblock_max(fl, S.ured);
    if (kmax >= static_cast<uint32_t>(kWin) && F < kmax - static_cast<uint32_t>(kWin - 1)) F = kmax - static_cast<uint32_t>(kWin - 1);
    for (int b = tid; b < kWin; b += kMT) S.cnt[b] = 0u;
    __syncthreads();
    for (int i = tid; i < total; i += kMT) {
      const unsigned key = static_cast<unsigned>(S.c[i] >> 32);
      if (key >= F) atomicAdd(&S.cnt[kmax - key], 1u);
    }
    __syncthreads();
    if (topk) {
      if (tid < 32) {
        unsigned tot = 0u;
        for (int b = lane; b < kWin; b += 32) tot += S.cnt[b];
        tot = __reduce_add_sync(0xFFFFFFFFu, tot);
        int b; unsigned above;
        warp_select_seq<unsigned, kWin, false>(S.cnt, static_cast<unsigned>(k_eff), &b, &above);
        if (lane == 0) {
          int good = tot >= static_cast<unsigned>(k_eff);
          uint32_t klk = 0u;
          if (good) {
            klk = tie_floor<DT, 16>(kmax - static_cast<uint32_t>(b), T);
            good = klk >= F;
          }
          S.ib[1] = good;
          S.ib[2] = static_cast<int>(klk);
        }
      }
      __syncthreads();
      ok = S.ib[1] != 0;
      key_lo_k = static_cast<uint32_t>(S.ib[2]);
    } else {
      ok = false;  // without top-k the slices' lists do not hold the row
    }
    key_lo = key_lo_k;
    if (ok && topp) {
      const int bk = static_cast<int>(kmax - key_lo_k);
      float* mb = reinterpret_cast<float*>(S.cnt);
      for (int b = tid; b < kWin; b += kMT) {
        const unsigned cn = S.cnt[b];
        mb[b] = (b <= bk && cn) ? __fmul_rn(static_cast<float>(cn), mass_of(C::value(kmax - static_cast<uint32_t>(b)), T, rT, M)) : 0.f;
      }
      __syncthreads();
      if (tid < 32) {
        float s = 0.f;
        for (int b = lane; b < kWin; b += 32) s += mb[b];
        s = warp_sum(s);
        const float target = __fmul_rn(pp, s);
        int b; float above;
        warp_select_seq<float, kWin, false>(mb, target, &b, &above);
        if (lane == 0) S.ib[3] = static_cast<int>(max(tie_floor<DT, 16>(kmax - static_cast<uint32_t>(b), T), key_lo_k));
      }
      __syncthreads();
      key_lo = static_cast<uint32_t>(S.ib[3]);
    }
    if (ok) {
      // inverse CDF over the merged entries in vocab order (thread t: a contiguous stretch)
      const uint32_t kdraw = max(key_lo, key_cut);
      const int per = (total + kMT - 1) / kMT;
      const int i0 = min(total, tid * per), i1 = min(total, i0 + per);
      float acc = 0.f;
      int lastp = -1;
      for (int i = i0; i < i1; ++i) {
        const unsigned key = static_cast<unsigned>(S.c[i] >> 32);
        if (key >= kdraw) {
          const float e = mass_of(C::value(key), T, rT, M);
          acc += e;
          if (e > 0.f) lastp = i;
        }
      }
      float incl = acc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane == 31) S.red[tid >> 5] = incl;
      __syncthreads();
      float base = 0.f, tot = 0.f;
      for (int w = 0; w < kMW; ++w) {
        if (w < (tid >> 5)) base += S.red[w];
        tot += S.red[w];
      }
      Z = tot;
      const float target = __fmul_rn(u, tot);
      const float ex = base + (incl - acc);
      int mine = INT_MAX;
      if (acc > 0.f && ex + acc > target) {
        float run = ex;
        for (int i = i0; i < i1 && mine == INT_MAX; ++i) {
          const unsigned key = static_cast<unsigned>(S.c[i] >> 32);
          if (key >= kdraw) {
            const float e = mass_of(C::value(key), T, rT, M);
            if (e > 0.f) { run += e; if (run > target) mine = i; }
          }
        }
        if (mine == INT_MAX) mine = lastp;
      }
      __syncthreads();
      const unsigned pick = mblock_min(static_cast<unsigned>(mine), S.ured);
      const unsigned last = mblock_max(static_cast<unsigned>(lastp + 1), S.ured);
      if (pick != static_cast<unsigned>(INT_MAX)) result = static_cast<int>(S.c[pick] & 0xFFFFFFFFu);
      else if (last > 0u) result = static_cast<int>(S.c[last - 1u] & 0xFFFFFFFFu);
      else ok = false;
    }
  }

  if (tid == 0) {
    P.out[row] = (greedy || ok) ? min(result, P.V - 1) : -1;
    if (P.row_stats) {
      float* st = P.row_stats + 4ll * row;
      if (greedy) { st[0] = ymax; st[1] = ymax; st[2] = ymax; st[3] = 1.0f; }
      else {
        st[0] = topk ? C::value(key_lo_k) : -INFINITY;
        st[1] = (topk || topp) ? C::value(key_lo) : -INFINITY;
        st[2] = M;
        st[3] = Z;
      }
    }
    if (!P.uniforms && P.philox_state) {
      // the last row to finish advances the Philox offset
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

}  // namespace vp
}  // namespace ecah
