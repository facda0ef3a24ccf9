// Fused token sampler for sm_100a.
//
// One thread-block cluster per batch row.  Each CTA of the cluster owns a
// contiguous chunk of the vocabulary and keeps it resident in shared memory
// as order-preserving keys of the penalised logit y' (16-bit keys when y'
// stays in the fp16/bf16 model dtype, 32-bit otherwise).  The logits are read
// from HBM exactly once; every later phase works on the resident keys and
// exchanges only per-CTA summaries (row max, 256-bin histograms, masses)
// through distributed shared memory.
//
// Phases per row (reference op order, ecahlang/main.py:169-170 then
// flashinfer top_k_top_p_sampling_from_logits, top_k_first):
//   1. load + key encode; sparse repetition / frequency / presence patch
//   2. row max of y' (cluster max)          -> M = y'_max / T
//   3. top-k threshold: radix select on the keys with count histograms
//   4. top-p threshold: radix select with softmax-mass histograms
//   5. inverse-CDF draw over the kept keys in vocab order
// Selection happens in y'-key space: z = y'/T is monotone in y', so the k-th
// largest z is (k-th largest y')/T, and a z threshold maps back to the least
// key whose quotient reaches it (key_lower_bound), which keeps ties that the
// float32 divide creates.  Only masses need the per-token divide.

#include <cooperative_groups.h>

#include <climits>
#include <cstdio>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace ecah {

struct KParams {
  const void* logits;
  long long row_stride;
  int B, V;
  const float* temperature;
  const int* top_k;
  const float* top_p;
  const float* rep_factor;
  const float* freq_pen;
  const float* pres_pen;
  const int* row_slot;
  const int* slot_len;
  const int* hist_tok;
  const int* hist_cnt;
  const float* hist_mval;
  int hist_cap;
  int num_slots;
  unsigned flags;
  const float* uniforms;
  unsigned long long* philox_state;
  int* out;
  float* row_stats;
  float* probs_out;
  unsigned* done_counter;  // workspace word for the Philox offset bump
  int CL;                  // CTAs per row (cluster size)
  int CH;                  // vocab entries per CTA (multiple of the vector width)
  int vec_ok;              // 16-byte aligned rows
};

struct Published {  // per-CTA values read by the other CTAs of the cluster
  unsigned kmax;
  int first_idx;
  float total;
};

// Smallest key k in [0, hi] whose quotient value(k)/T reaches zthr.  The
// predicate is monotone over [0, hi] (NaN keys sit below -inf; hi is never a
// NaN key) and callers guarantee it holds at hi.  32-bit keys gallop from the
// guess key(zthr*T) before bisecting; 16-bit keys bisect directly.
template <class C>
__device__ uint32_t key_lower_bound(float zthr, float T, uint32_t hi) {
  auto pred = [&](uint32_t k) { return __fdiv_rn(C::value(k), T) >= zthr; };
  if (!pred(hi)) return hi;
  uint32_t lo = 0u, h = hi;  // answer in [lo, h]; pred(h) holds
  if constexpr (C::kBits == 32) {
    const float gv = __fmul_rn(zthr, T);
    uint32_t g = (gv != gv) ? 0u : key32(gv);
    if (g > hi) g = hi;
    if (pred(g)) {
      h = g;
      for (uint64_t step = 1;; step <<= 1) {
        if (step > g) { lo = 0u; break; }
        const uint32_t c = g - static_cast<uint32_t>(step);
        if (!pred(c)) { lo = c + 1u; break; }
        h = c;
      }
    } else {
      lo = g + 1u;
      for (uint64_t step = 1;; step <<= 1) {
        if (step >= static_cast<uint64_t>(hi - g)) break;  // h stays hi
        const uint32_t c = g + static_cast<uint32_t>(step);
        if (pred(c)) { h = c; break; }
        lo = c + 1u;
      }
    }
  }
  while (lo < h) {
    const uint32_t mid = lo + ((h - lo) >> 1);
    if (pred(mid)) h = mid; else lo = mid + 1u;
  }
  return lo;
}

// Warp-0 selection over 256 bins in descending bin order: the first bin at
// which the running total reaches `target`.  Returns bin and the total of the
// bins above it.  If rounding leaves the target unreached, the lowest bin with
// a non-zero value is taken (the most inclusive choice).
template <typename T>
__device__ void select_bin_desc(const T* hist, T target, int* out_bin, T* out_above) {
  const int lane = threadIdx.x & 31;
  T v[8];
  T s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = hist[255 - 8 * lane - j];
    s += v[j];
  }
  T incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  T excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
  if (lane == 0) excl = 0;
  unsigned hit = __ballot_sync(0xFFFFFFFFu, incl >= target);
  int bin = -1;
  T above = 0;
  if (hit) {
    const int L = __ffs(hit) - 1;
    if (lane == L) {
      T acc = excl;
      int last_nz = -1;
      T acc_last = 0;
      for (int j = 0; j < 8; ++j) {
        if (v[j] > 0) { last_nz = j; acc_last = acc; }
        if (acc + v[j] >= target && v[j] > 0) { bin = 255 - 8 * lane - j; above = acc; break; }
        acc += v[j];
      }
      if (bin < 0 && last_nz >= 0) { bin = 255 - 8 * lane - last_nz; above = acc_last; }
      if (bin < 0) { bin = 255 - 8 * lane - 7; above = acc; }
    }
    bin = __shfl_sync(0xFFFFFFFFu, bin, L);
    above = __shfl_sync(0xFFFFFFFFu, above, L);
  } else {
    // target beyond the total: lowest non-zero bin
    unsigned nz = __ballot_sync(0xFFFFFFFFu, s > 0);
    const int L = nz ? 31 - __clz(nz) : 31;
    if (lane == L) {
      T acc = excl;
      int jb = 7;
      for (int j = 7; j >= 0; --j) if (v[j] > 0) { jb = j; break; }
      for (int j = 0; j < jb; ++j) acc += v[j];
      bin = 255 - 8 * lane - jb;
      above = acc;
    }
    bin = __shfl_sync(0xFFFFFFFFu, bin, L);
    above = __shfl_sync(0xFFFFFFFFu, above, L);
  }
  if (lane == 0) { *out_bin = bin; *out_above = above; }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

template <int DT, int KB>
__global__ void __launch_bounds__(kThreads, 2) sample_kernel(const KParams P) {
  using Dt = DType<DT>;
  using C = Codec<DT, KB>;
  using Key = typename C::Key;
  using Raw = typename Dt::Raw;
  constexpr int VEC = Dt::kVec;                    // logits per 16-byte global load
  constexpr int SEG = 32 * VEC;                    // keys per warp segment

  extern __shared__ __align__(16) unsigned char dsm[];
  Key* keys = reinterpret_cast<Key*>(dsm);

  __shared__ unsigned s_cnt[2][256];
  __shared__ float s_mass[2][256];
  __shared__ unsigned s_mcnt[256];
  __shared__ float s_mmass[256];
  __shared__ float s_seg[1024];
  __shared__ unsigned s_red[kWarps];
  __shared__ Published s_pub;
  __shared__ int s_bin;
  __shared__ unsigned s_above_u;
  __shared__ float s_above_f;
  __shared__ int s_sel[4];
  __shared__ float s_self[4];

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int row = blockIdx.x / P.CL;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = rank * P.CH;
  const int n = max(0, min(P.CH, P.V - c0));
  const int nvec = (n + VEC - 1) / VEC;
  const Raw* src = reinterpret_cast<const Raw*>(P.logits) + static_cast<long long>(row) * P.row_stride + c0;

  for (int i = tid; i < 512; i += kThreads) { (&s_cnt[0][0])[i] = 0u; (&s_mass[0][0])[i] = 0.f; }

  // ------------------------------------------------------------ 1. load
  const int nfull = n / VEC;
  if (P.vec_ok) {
    for (int v = tid; v < nfull; v += kThreads) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(src) + v);
      if constexpr (VEC == 8 && KB == 16) {
        uint4 k;
        k.x = key16x2(w.x); k.y = key16x2(w.y); k.z = key16x2(w.z); k.w = key16x2(w.w);
        reinterpret_cast<uint4*>(keys)[v] = k;
      } else if constexpr (VEC == 8) {
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        uint4 a, b;
        uint32_t* pa = &a.x;
        uint32_t* pb = &b.x;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          pa[2 * j] = C::from_raw(ws[j] & 0xFFFFu);
          pa[2 * j + 1] = C::from_raw(ws[j] >> 16);
          pb[2 * j] = C::from_raw(ws[j + 2] & 0xFFFFu);
          pb[2 * j + 1] = C::from_raw(ws[j + 2] >> 16);
        }
        reinterpret_cast<uint4*>(keys)[2 * v] = a;
        reinterpret_cast<uint4*>(keys)[2 * v + 1] = b;
      } else {
        uint4 k;
        k.x = C::from_raw(w.x); k.y = C::from_raw(w.y); k.z = C::from_raw(w.z); k.w = C::from_raw(w.w);
        reinterpret_cast<uint4*>(keys)[v] = k;
      }
    }
    for (int i = nfull * VEC + tid; i < n; i += kThreads) keys[i] = static_cast<Key>(C::from_raw(src[i]));
  } else {
    for (int i = tid; i < n; i += kThreads) keys[i] = static_cast<Key>(C::from_raw(src[i]));
  }

  // per-row parameters
  const float T = P.temperature[row];
  int kk = P.top_k[row];
  const int k_eff = (kk <= 0 || kk >= P.V) ? P.V : kk;
  const float pp = P.top_p[row];
  const bool topp_on = (pp > 0.f && pp < 1.f);
  float u;
  if (P.uniforms) {
    u = P.uniforms[row];
  } else {
    const unsigned long long seed = P.philox_state[0], off = P.philox_state[1];
    u = row_uniform(seed, off, static_cast<uint64_t>(row));
  }
  __syncthreads();

  // ---------------------------------------------------- 1b. penalty patch
  if (P.row_slot) {
    const int slot = P.row_slot[row];
    if (slot >= 0 && slot < P.num_slots) {
      const int len = min(P.slot_len[slot], P.hist_cap);
      const float rf = P.rep_factor ? P.rep_factor[row] : 1.0f;
      const bool fp = (P.flags & ECAH_FLAG_FREQ_PRES) != 0;
      const float fq = (fp && P.freq_pen) ? P.freq_pen[row] : 0.f;
      const float pr = (fp && P.pres_pen) ? P.pres_pen[row] : 0.f;
      const long long base = static_cast<long long>(slot) * P.hist_cap;
      for (int h = tid; h < len; h += kThreads) {
        const int tok = P.hist_tok[base + h];
        const int cnt = P.hist_cnt[base + h];
        const int li = tok - c0;
        if (cnt <= 0 || li < 0 || li >= n) continue;
        const float x = Dt::to_f32(src[li]);
        const float m = P.hist_mval ? P.hist_mval[base + h] : penalty_divisor<DT>(cnt, rf);
        float y = Dt::round(__fdiv_rn(x, m));
        if (fp) y = __fsub_rn(y, __fadd_rn(__fmul_rn(fq, static_cast<float>(cnt)), pr));
        keys[li] = static_cast<Key>(C::from_val(y));
      }
    }
  }
  __syncthreads();

  // ------------------------------------------------------------- 2. max
  unsigned tmax = 0;
  for (int i = tid; i < n; i += kThreads) tmax = max(tmax, static_cast<unsigned>(keys[i]));
  tmax = __reduce_max_sync(0xFFFFFFFFu, tmax);
  if (lane == 0) s_red[warp] = tmax;
  __syncthreads();
  if (tid == 0) {
    unsigned m = 0;
    for (int w = 0; w < kWarps; ++w) m = max(m, s_red[w]);
    s_pub.kmax = (n > 0) ? m : 0u;
  }
  cluster.sync();
  unsigned kmax = 0;
  for (int r = 0; r < P.CL; ++r) kmax = max(kmax, cluster.map_shared_rank(&s_pub, r)->kmax);

  const float ymax = C::value(kmax);
  const float M = __fdiv_rn(ymax, T);
  const bool greedy = !(T > 0.f) || !isfinite(M);

  int result = -1;  // written by the CTA that owns the sampled token

  if (greedy) {
    // argmax with the lowest index
    int first = INT_MAX;
    for (int i = tid; i < n; i += kThreads)
      if (static_cast<unsigned>(keys[i]) == kmax) { first = i; break; }
    first = __reduce_min_sync(0xFFFFFFFFu, first);
    if (lane == 0) s_red[warp] = static_cast<unsigned>(first);
    __syncthreads();
    if (tid == 0) {
      int f = INT_MAX;
      for (int w = 0; w < kWarps; ++w) f = min(f, static_cast<int>(s_red[w]));
      s_pub.first_idx = (f == INT_MAX) ? INT_MAX : f + c0;
    }
    cluster.sync();
    if (tid == 0) {
      int f = INT_MAX;
      for (int r = 0; r < P.CL; ++r) f = min(f, cluster.map_shared_rank(&s_pub, r)->first_idx);
      f = (f == INT_MAX) ? 0 : f;
      s_sel[0] = f;
      if (rank == 0) result = f;
    }
    if (P.row_stats && rank == 0 && tid == 0) {
      float* st = P.row_stats + 4ll * row;
      st[0] = ymax; st[1] = ymax; st[2] = ymax; st[3] = 1.0f;
    }
    if (P.probs_out) {
      __syncthreads();
      const int g = s_sel[0] - c0;
      float* po = P.probs_out + static_cast<long long>(row) * P.V + c0;
      for (int i = tid; i < n; i += kThreads) po[i] = (i == g) ? 1.0f : 0.0f;
    }
  } else {
    // key_cut: tokens below it have mass exactly zero
    const uint32_t key_cut = key_lower_bound<C>(__fsub_rn(M, kExpCut), T, kmax);
    uint32_t key_lo = 0;  // kept set: key >= key_lo
    uint32_t key_lo_k = 0;

    // ------------------------------------------------------- 3. top-k
    if (k_eff < P.V) {
      uint32_t prefix = 0;
      unsigned krem = static_cast<unsigned>(k_eff);
      for (int lev = 0; lev < KB / 8; ++lev) {
        const int shift = KB - 8 * (lev + 1);
        unsigned* h = s_cnt[lev & 1];
        if (lev > 0) {
          for (int i = tid; i < 256; i += kThreads) h[i] = 0u;
          __syncthreads();
        }
        if (lev == 0) {
          for (int i = tid; i < n; i += kThreads) atomicAdd(&h[static_cast<unsigned>(keys[i]) >> shift], 1u);
        } else {
          for (int i = tid; i < n; i += kThreads) {
            const unsigned k = keys[i];
            if ((k >> (shift + 8)) == prefix) atomicAdd(&h[(k >> shift) & 255u], 1u);
          }
        }
        cluster.sync();
        {
          unsigned s = 0;
          for (int r = 0; r < P.CL; ++r) s += cluster.map_shared_rank(h, r)[tid];
          s_mcnt[tid] = s;
        }
        __syncthreads();
        if (warp == 0) {
          int bin; unsigned above;
          select_bin_desc<unsigned>(s_mcnt, krem, &bin, &above);
          if (lane == 0) { s_bin = bin; s_above_u = above; }
        }
        __syncthreads();
        prefix = (prefix << 8) | static_cast<uint32_t>(s_bin);
        krem -= s_above_u;
      }
      // prefix = the k-th largest key; keep every key whose quotient ties it
      key_lo = key_lower_bound<C>(__fdiv_rn(C::value(prefix), T), T, prefix);
      key_lo_k = key_lo;
    }

    // ------------------------------------------------------- 4. top-p
    if (topp_on) {
      const uint32_t klo = max(key_lo, key_cut);
      uint32_t prefix = 0;
      float target = 0.f;
      for (int lev = 0; lev < KB / 8; ++lev) {
        const int shift = KB - 8 * (lev + 1);
        float* h = s_mass[lev & 1];
        if (lev > 0) {
          for (int i = tid; i < 256; i += kThreads) h[i] = 0.f;
          __syncthreads();
        }
        for (int i = tid; i < n; i += kThreads) {
          const unsigned k = keys[i];
          if (k < klo) continue;
          if (lev > 0 && (k >> (shift + 8)) != prefix) continue;
          atomicAdd(&h[(k >> shift) & 255u], token_mass(C::value(k), T, M));
        }
        cluster.sync();
        {
          float s = 0.f;
          for (int r = 0; r < P.CL; ++r) s += cluster.map_shared_rank(h, r)[tid];
          s_mmass[tid] = s;
        }
        __syncthreads();
        if (lev == 0) {
          // S over the top-k set, summed in a fixed order
          if (warp == 0) {
            float s = 0.f;
            for (int j = 0; j < 8; ++j) s += s_mmass[8 * lane + j];
            s = warp_sum(s);
            if (lane == 0) s_self[0] = s;
          }
          __syncthreads();
          target = __fmul_rn(pp, s_self[0]);
        }
        if (warp == 0) {
          int bin; float above;
          select_bin_desc<float>(s_mmass, target, &bin, &above);
          if (lane == 0) { s_bin = bin; s_above_f = above; }
        }
        __syncthreads();
        prefix = (prefix << 8) | static_cast<uint32_t>(s_bin);
        target = __fsub_rn(target, s_above_f);
        __syncthreads();
      }
      key_lo = key_lower_bound<C>(__fdiv_rn(C::value(prefix), T), T, prefix);
    }

    // ---------------------------------------------------------- 5. draw
    const uint32_t kdraw = max(key_lo, key_cut);
    const int nseg = (nvec + 31) / 32;
    for (int s = warp; s < nseg; s += kWarps) {
      const int e0 = s * SEG + lane * VEC;
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const int i = e0 + j;
        if (i < n) {
          const unsigned k = keys[i];
          if (k >= kdraw) acc += token_mass(C::value(k), T, M);
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) s_seg[s] = acc;
    }
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int s = 0; s < nseg; ++s) t += s_seg[s];
      s_pub.total = t;
    }
    cluster.sync();
    if (tid == 0) {
      float Z = 0.f;
      for (int r = 0; r < P.CL; ++r) Z += cluster.map_shared_rank(&s_pub, r)->total;
      const float target = __fmul_rn(u, Z);
      float run = 0.f;
      int rsel = -1, rlast = -1;
      float run_sel = 0.f, run_last = 0.f;
      for (int r = 0; r < P.CL; ++r) {
        const float tr = cluster.map_shared_rank(&s_pub, r)->total;
        if (tr > 0.f) { rlast = r; run_last = run; }
        if (rsel < 0 && tr > 0.f && run + tr > target) { rsel = r; run_sel = run; }
        run += tr;
      }
      bool take_last = false;
      if (rsel < 0) { rsel = rlast; run_sel = run_last; take_last = true; }
      s_sel[0] = rsel;
      s_sel[1] = take_last ? 1 : 0;
      s_self[1] = __fsub_rn(target, run_sel);
      s_self[3] = Z;
      if (P.row_stats && rank == 0) {
        float* st = P.row_stats + 4ll * row;
        st[0] = (k_eff < P.V) ? C::value(key_lo_k) : -INFINITY;
        st[1] = (k_eff < P.V || topp_on) ? C::value(key_lo) : -INFINITY;
        st[2] = M; st[3] = Z;
      }
    }
    __syncthreads();
    const int rsel = s_sel[0];
    if (rsel < 0) {
      // no mass anywhere (non-finite input): fall back to the row max
      if (rank == 0 && tid == 0) result = -2;
    } else if (rank == rsel) {
      bool take_last = s_sel[1] != 0;
      if (tid == 0) {
        const float rem = s_self[1];
        float run = 0.f, run_last = 0.f;
        int ssel = -1, slast = -1;
        for (int s = 0; s < nseg; ++s) {
          const float v = s_seg[s];
          if (v > 0.f) { slast = s; run_last = run; }
          if (!take_last && ssel < 0 && v > 0.f && run + v > rem) { ssel = s; s_self[2] = __fsub_rn(rem, run); }
          run += v;
        }
        if (ssel < 0) { ssel = slast; take_last = true; s_self[2] = 0.f; (void)run_last; }
        if (ssel < 0) ssel = 0;  // unreachable: the selected CTA has positive mass
        s_sel[2] = ssel;
        s_sel[3] = take_last ? 1 : 0;
      }
      __syncthreads();
      if (warp == 0) {
        const int s = s_sel[2];
        const bool last = s_sel[3] != 0;
        const float rem = s_self[2];
        const int e0 = s * SEG + lane * VEC;
        float ev[VEC];
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const int i = e0 + j;
          float e = 0.f;
          if (i < n) {
            const unsigned k = keys[i];
            if (k >= kdraw) e = token_mass(C::value(k), T, M);
          }
          ev[j] = e;
          acc += e;
        }
        float incl = acc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += y;
        }
        float excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
        if (lane == 0) excl = 0.f;
        unsigned hit = last ? 0u : __ballot_sync(0xFFFFFFFFu, acc > 0.f && incl > rem);
        int L;
        if (hit) {
          L = __ffs(hit) - 1;
        } else {
          const unsigned nz = __ballot_sync(0xFFFFFFFFu, acc > 0.f);
          L = nz ? 31 - __clz(nz) : 0;
        }
        if (lane == L) {
          int pick = -1, lastpos = -1;
          float run = excl;
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            if (ev[j] > 0.f) {
              lastpos = j;
              run += ev[j];
              if (!last && hit && pick < 0 && run > rem) pick = j;
            }
          }
          if (pick < 0) pick = lastpos;
          if (pick < 0) pick = 0;
          s_sel[0] = c0 + e0 + pick;
        }
        __syncwarp();
      }
      __syncthreads();
      if (tid == 0) result = s_sel[0];
    }
    if (rsel < 0) {
      // fallback: first index of the maximum key (cluster-wide)
      int first = INT_MAX;
      for (int i = tid; i < n; i += kThreads)
        if (static_cast<unsigned>(keys[i]) == kmax) { first = i; break; }
      first = __reduce_min_sync(0xFFFFFFFFu, first);
      if (lane == 0) s_red[warp] = static_cast<unsigned>(first);
      __syncthreads();
      if (tid == 0) {
        int f = INT_MAX;
        for (int w = 0; w < kWarps; ++w) f = min(f, static_cast<int>(s_red[w]));
        s_pub.first_idx = (f == INT_MAX) ? INT_MAX : f + c0;
      }
      cluster.sync();
      if (rank == 0 && tid == 0) {
        int f = INT_MAX;
        for (int r = 0; r < P.CL; ++r) f = min(f, cluster.map_shared_rank(&s_pub, r)->first_idx);
        result = (f == INT_MAX) ? 0 : f;
      }
    }
    if (P.probs_out) {
      // the renormalised distribution the draw used (same masses, same Z)
      const float Z = s_self[3];
      float* po = P.probs_out + static_cast<long long>(row) * P.V + c0;
      for (int i = tid; i < n; i += kThreads) {
        const unsigned k = keys[i];
        po[i] = (k >= kdraw && rsel >= 0) ? __fdiv_rn(token_mass(C::value(k), T, M), Z) : 0.0f;
      }
    }
  }

  if (tid == 0 && result >= 0) P.out[row] = min(result, P.V - 1);

  // keep this CTA's shared memory alive until every peer is done reading it
  cluster.sync();

  if (!P.uniforms && rank == 0 && tid == 0) {
    // the last cluster to finish advances the Philox offset; every cluster has
    // read the offset before it arrives here
    __threadfence();
    const unsigned prev = atomicAdd(P.done_counter, 1u);
    if (prev == static_cast<unsigned>(P.B) - 1u) {
      P.philox_state[1] += 1ull;
      *P.done_counter = 0u;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------- hist update
template <int DT>
__global__ void hist_update_kernel(const int* ids, int B, const int* row_slot, const float* rep_factor,
                                   int* slot_len, int* hist_tok, int* hist_cnt, float* hist_mval, int cap,
                                   int num_slots, int* overflow) {
  const int warps = blockDim.x / 32;
  const int r = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= B) return;
  const int slot = row_slot[r];
  if (slot < 0 || slot >= num_slots) return;
  const int tok = ids[r];
  const float rf = rep_factor ? rep_factor[r] : 1.0f;
  const long long base = static_cast<long long>(slot) * cap;
  const int len = min(slot_len[slot], cap);
  int found = -1;
  for (int j0 = 0; j0 < len && found < 0; j0 += 32) {
    const int j = j0 + lane;
    const bool hit = (j < len) && hist_tok[base + j] == tok;
    const unsigned b = __ballot_sync(0xFFFFFFFFu, hit);
    if (b) found = j0 + __ffs(b) - 1;
  }
  if (lane != 0) return;
  if (found >= 0) {
    hist_cnt[base + found] += 1;
    hist_mval[base + found] = penalty_step<DT>(hist_mval[base + found], rf);
  } else if (len < cap) {
    hist_tok[base + len] = tok;
    hist_cnt[base + len] = 1;
    hist_mval[base + len] = penalty_step<DT>(1.0f, rf);
    slot_len[slot] = len + 1;
  } else if (overflow) {
    overflow[slot] = 1;
  }
}

__global__ void philox_uniforms_kernel(unsigned long long* state, int B, float* out, int advance) {
  const unsigned long long seed = state[0], off = state[1];
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < B; r += gridDim.x * blockDim.x)
    out[r] = row_uniform(seed, off, static_cast<uint64_t>(r));
  // single-block launch: every thread has read the state before this point
  __syncthreads();
  if (advance && threadIdx.x == 0) state[1] = off + 1ull;
}

// ----------------------------------------------------------------- host side
using KernelFn = void (*)(const KParams);

template <int DT, int KB>
static KernelFn kernel_for() { return sample_kernel<DT, KB>; }

static KernelFn pick_kernel(int dtype, int kb) {
  if (dtype == ECAH_DTYPE_F16) return kb == 16 ? kernel_for<ECAH_DTYPE_F16, 16>() : kernel_for<ECAH_DTYPE_F16, 32>();
  if (dtype == ECAH_DTYPE_BF16) return kb == 16 ? kernel_for<ECAH_DTYPE_BF16, 16>() : kernel_for<ECAH_DTYPE_BF16, 32>();
  return kernel_for<ECAH_DTYPE_F32, 32>();
}

static int elem_size(int dtype) { return dtype == ECAH_DTYPE_F32 ? 4 : 2; }

struct Plan {
  int CL, CH, kb;
  size_t smem;
};

static constexpr size_t kMaxDynSmem = 200 * 1024;

static bool make_plan(int dtype, int V, unsigned flags, Plan* p) {
  const int kb = (dtype == ECAH_DTYPE_F32 || (flags & ECAH_FLAG_FREQ_PRES)) ? 32 : 16;
  const int vec = dtype == ECAH_DTYPE_F32 ? 4 : 8;
  const int ksz = kb / 8;
  const int target = (kb == 16) ? 20480 : 12288;  // keys per CTA aimed for
  int CL = (V + target - 1) / target;
  if (CL < 1) CL = 1;
  if (CL > 8) CL = (CL <= 16) ? 16 : CL;
  if (CL > 16) CL = 16;
  int CH = (V + CL - 1) / CL;
  CH = (CH + vec - 1) / vec * vec;
  size_t smem = static_cast<size_t>(CH) * ksz;
  smem = (smem + 15) / 16 * 16;
  if (smem > kMaxDynSmem) return false;
  if ((CH + 32 * vec - 1) / (32 * vec) > 1024) return false;
  p->CL = CL; p->CH = CH; p->kb = kb; p->smem = smem;
  return true;
}

}  // namespace ecah

using namespace ecah;

extern "C" {

int ecah_sampler_abi_version(void) { return ECAH_SAMPLER_ABI_VERSION; }

const char* ecah_status_string(int s) {
  switch (s) {
    case ECAH_OK: return "ok";
    case ECAH_ERR_NULL: return "a required pointer is NULL";
    case ECAH_ERR_DTYPE: return "unsupported dtype";
    case ECAH_ERR_SHAPE: return "batch/vocab/row_stride out of range";
    case ECAH_ERR_WORKSPACE: return "workspace missing or too small";
    case ECAH_ERR_LAUNCH: return "CUDA launch failed";
    case ECAH_ERR_ABI: return "abi_version mismatch";
    default: return "unknown status";
  }
}

size_t ecah_sampler_workspace_bytes(int32_t batch, int32_t vocab, int32_t dtype) {
  (void)batch; (void)vocab; (void)dtype;
  return 256;
}

int ecah_sampler_launch(const ecah_sampler_args* a, void* stream) {
  if (!a) return ECAH_ERR_NULL;
  if (a->abi_version != ECAH_SAMPLER_ABI_VERSION) return ECAH_ERR_ABI;
  if (a->dtype < ECAH_DTYPE_F16 || a->dtype > ECAH_DTYPE_F32) return ECAH_ERR_DTYPE;
  if (a->batch < 0 || a->vocab < 1 || a->row_stride < a->vocab) return ECAH_ERR_SHAPE;
  if (a->batch == 0) return ECAH_OK;
  if (!a->logits || !a->temperature || !a->top_k || !a->top_p || !a->out) return ECAH_ERR_NULL;
  if (!a->uniforms && !a->philox_state) return ECAH_ERR_NULL;
  if (a->row_slot && (!a->slot_len || !a->hist_tok || !a->hist_cnt || a->hist_cap < 0)) return ECAH_ERR_NULL;
  if (!a->workspace || a->workspace_bytes < ecah_sampler_workspace_bytes(a->batch, a->vocab, a->dtype))
    return ECAH_ERR_WORKSPACE;
  Plan plan;
  if (!make_plan(a->dtype, a->vocab, a->flags, &plan)) return ECAH_ERR_SHAPE;
  if (static_cast<long long>(a->batch) * plan.CL > 0x7FFFFFFFLL) return ECAH_ERR_SHAPE;

  KParams P;
  P.logits = a->logits;
  P.row_stride = a->row_stride;
  P.B = a->batch;
  P.V = a->vocab;
  P.temperature = a->temperature;
  P.top_k = a->top_k;
  P.top_p = a->top_p;
  P.rep_factor = a->rep_factor;
  P.freq_pen = a->freq_pen;
  P.pres_pen = a->pres_pen;
  P.row_slot = a->row_slot;
  P.slot_len = a->slot_len;
  P.hist_tok = a->hist_tok;
  P.hist_cnt = a->hist_cnt;
  P.hist_mval = a->hist_mval;
  P.hist_cap = a->hist_cap;
  P.num_slots = a->num_slots;
  P.flags = a->flags;
  P.uniforms = a->uniforms;
  P.philox_state = reinterpret_cast<unsigned long long*>(a->philox_state);
  P.out = a->out;
  P.row_stats = a->row_stats;
  P.probs_out = a->probs_out;
  P.done_counter = reinterpret_cast<unsigned*>(a->workspace);
  P.CL = plan.CL;
  P.CH = plan.CH;
  const int es = elem_size(a->dtype);
  P.vec_ok = (reinterpret_cast<uintptr_t>(a->logits) % 16 == 0) && ((a->row_stride * es) % 16 == 0);

  KernelFn fn = pick_kernel(a->dtype, plan.kb);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan.smem));
  if (e != cudaSuccess) return ECAH_ERR_LAUNCH;
  if (plan.CL > 8) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return ECAH_ERR_LAUNCH;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a->batch * plan.CL), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = plan.CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, fn, P);
  return e == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

int ecah_hist_update(const int32_t* ids, int32_t batch, const int32_t* row_slot, const float* rep_factor,
                     int32_t* slot_len, int32_t* hist_tok, int32_t* hist_cnt, float* hist_mval, int32_t hist_cap,
                     int32_t num_slots, int32_t dtype, int32_t* overflow, void* stream) {
  if (batch < 0 || hist_cap < 0 || num_slots < 0) return ECAH_ERR_SHAPE;
  if (batch == 0) return ECAH_OK;
  if (!ids || !row_slot || !slot_len || !hist_tok || !hist_cnt || !hist_mval) return ECAH_ERR_NULL;
  const int threads = 256, rows_per_block = threads / 32;
  const dim3 grid((batch + rows_per_block - 1) / rows_per_block);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case ECAH_DTYPE_F16:
      hist_update_kernel<ECAH_DTYPE_F16><<<grid, threads, 0, s>>>(ids, batch, row_slot, rep_factor, slot_len, hist_tok,
                                                                 hist_cnt, hist_mval, hist_cap, num_slots, overflow);
      break;
    case ECAH_DTYPE_BF16:
      hist_update_kernel<ECAH_DTYPE_BF16><<<grid, threads, 0, s>>>(ids, batch, row_slot, rep_factor, slot_len,
                                                                  hist_tok, hist_cnt, hist_mval, hist_cap, num_slots, overflow);
      break;
    case ECAH_DTYPE_F32:
      hist_update_kernel<ECAH_DTYPE_F32><<<grid, threads, 0, s>>>(ids, batch, row_slot, rep_factor, slot_len, hist_tok,
                                                                 hist_cnt, hist_mval, hist_cap, num_slots, overflow);
      break;
    default:
      return ECAH_ERR_DTYPE;
  }
  return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

int ecah_philox_uniforms(uint64_t* philox_state, int32_t batch, float* out, int32_t advance, void* stream) {
  if (batch < 0) return ECAH_ERR_SHAPE;
  if (!philox_state || (!out && batch > 0)) return ECAH_ERR_NULL;
  philox_uniforms_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<unsigned long long*>(philox_state), batch, out, advance);
  return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

}  // extern "C"
