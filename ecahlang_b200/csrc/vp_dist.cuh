// Vocab-parallel rows without top-k (the reference's default request, top_k =
// V, and top-p-only rows): the exact distributed sampler, one pass over this
// rank's slice per call (ecah_vp_dist_pass).  The caller reduces each pass's
// per-row outputs over the ranks between passes (NCCL) and hands the results
// to vp_dist_combine_kernel, which turns them into the per-row state the next
// pass reads ([n, kState] floats), so every decision stays on the device:
//   pass 1  per row: z of the slice max, the lowest global id holding it, and
//           the slice's mass relative to that max.  Combine: M = the row max;
//           without top-p every entry above the zero-mass cut is kept, so
//           the slices' masses rescaled to M already name the rank that owns
//           the draw (passes 2-4 skip the row)
//   pass 2  mass (relative to M) per high key byte                    [256]
//   pass 3  inside high byte hb: mass per low key byte, plus the mass of the
//           keys above hb                                             [257]
//           Combine: the top-p threshold key, the reference's rule (the
//           largest z whose mass from the top reaches top_p * Z)
//   pass 4  the slice's kept mass (keys >= kdraw; kdraw from the threshold
//           key through tie_floor and the zero-mass cut).  Combine: the
//           owning rank and its local target
//   pass 5  on the owning rank: the lowest global id whose inclusive
//           cumulative kept mass in vocab order exceeds its target; -1 on
//           the other ranks (all-reduced with max)
// Masses are mass_of of the penalised logit (the semantics of every kernel
// here).  One CTA of kDT threads per listed row; the slice is staged in
// chunks of kDCH entries with the penalty patch applied (history ids are
// global).  Rows listed that have a top-k (1 <= top_k < vocab) or T <= 0 are
// the candidate path's: every pass skips them and their ids are left as they
// are.
#pragma once

#include "sampler_kernel.cuh"
#include "stream_kernel.cuh"

namespace ecah {
namespace vd {

constexpr int kDT = 256;
constexpr int kDCH = 4096;               // entries per staged chunk (two buffers)
constexpr int kDPer = kDCH / kDT;        // 16 consecutive entries per thread

// per-row state between passes
constexpr int kState = 8;
enum : int { kSM = 0, kSHb = 1, kSTau = 2, kST = 3, kSTarget = 4, kSFlag = 5 };
// kSHb: -1 no top-p, kOwnerKnown no top-p and the draw's owner already chosen
// from the pass-1 masses (passes 2-4 skip the row), else the high key byte
constexpr float kOwnerKnown = -2.f;
// kSFlag: 0 served, 1 not this path's row (left untouched), 2 refused (id -1:
// a NaN logit, or no mass)

// the rows this path serves: sampled (T > 0) with top-k off
__device__ __forceinline__ bool full_row(const float* temperature, const int* top_k, int vocab, int row) {
  const int k = top_k[row];
  return temperature[row] > 0.f && (k <= 0 || k >= vocab);
}

struct DParams {
  KParams P;                             // slice, parameters, histories (row_kernel's fields)
  int pass;
  const int* rows;                       // [n] rows of the batch to serve
  int n;
  const float* gin;                      // [n, kState] the row state (passes 2-5)
  float* gout;                           // [n, width] outputs (pass 5: int ids)
};

// Pipelined staging: the vector part of the next chunk is copied in (cp.async,
// one commit group per chunk) while the current chunk is counted; two
// buffers alternate.  stage_issue starts chunk [c0, c0 + len) into buf;
// stage_finish waits for it (the next chunk's group may stay in flight),
// then loads the scalar rest, pads past the slice end and applies the
// penalty patch, as stage does.
template <int DT>
__device__ __forceinline__ void stage_issue(const KParams& P, uint16_t* buf, int row, int c0, int len) {
  if (P.vec_ok && len > 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(P.logits) + logits_row_offset(P, row) + c0);
    uint4* r4 = reinterpret_cast<uint4*>(buf);
    const int nv = len >> 3;
    for (int v = threadIdx.x; v < nv; v += kDT) cp_async16(r4 + v, s4 + v);
  }
  cp_async_commit();
}

template <int DT>
__device__ void stage_finish(const KParams& P, uint16_t* raw, int row, int c0, int len) {
  cp_async_wait_group<1>();
  const uint16_t* src = static_cast<const uint16_t*>(P.logits) + logits_row_offset(P, row) + c0;
  const int done = P.vec_ok ? ((len >> 3) << 3) : 0;
  for (int i = done + threadIdx.x; i < kDCH; i += kDT) raw[i] = (i < len) ? src[i] : static_cast<uint16_t>(0xFFFFu);
  __syncthreads();
  if (P.row_slot) {
    const int slot = P.row_slot[row];
    if (slot >= 0 && slot < P.num_slots) {
      const int hl = min(P.slot_len[slot], P.hist_cap);
      const float rf = P.rep_factor ? P.rep_factor[row] : 1.0f;
      const long long base = static_cast<long long>(slot) * P.hist_cap;
      for (int h = threadIdx.x; h < hl; h += kDT) {
        const int li = P.hist_tok[base + h] - P.vocab_offset - c0;
        const int cnt = P.hist_cnt[base + h];
        if (cnt <= 0 || li < 0 || li >= len) continue;
        const float m = P.hist_mval ? P.hist_mval[base + h] : penalty_divisor<DT>(cnt, rf);
        raw[li] = static_cast<uint16_t>(DType<DT>::to_raw(penalise<DT>(DType<DT>::to_f32(raw[li]), m, 0.f)));
      }
    }
    __syncthreads();
  }
}

// the chunk loop: fn(raw, c0, len) counts a staged chunk; it returns false
// to stop early (every thread the same), after which no copy stays in flight
template <int DT, typename Fn>
__device__ __forceinline__ void stream_slice(const KParams& P, uint16_t (*bufs)[kDCH], int row, int V, Fn&& fn) {
  stage_issue<DT>(P, bufs[0], row, 0, min(kDCH, V));
  int k = 0;
  for (int c0 = 0; c0 < V; c0 += kDCH, ++k) {
    const int len = min(kDCH, V - c0);
    if (c0 + kDCH < V) stage_issue<DT>(P, bufs[(k + 1) & 1], row, c0 + kDCH, min(kDCH, V - c0 - kDCH));
    else cp_async_commit();   // an empty group keeps the count of groups in flight
    stage_finish<DT>(P, bufs[k & 1], row, c0, len);
    const bool more = fn(bufs[k & 1], c0, len);
    __syncthreads();          // the buffer is refilled two chunks on
    if (!more) break;
  }
  cp_async_wait_group<0>();
}

__device__ __forceinline__ float bsum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kDT / 32; ++i) t += red[i];
  return t;
}

template <int DT>
__global__ void __launch_bounds__(kDT) vp_dist_kernel(const __grid_constant__ DParams D) {
  using C = Codec<DT, 16>;
  using Dt = DType<DT>;
  __shared__ __align__(16) uint16_t rawb[2][kDCH];
  __shared__ float hist[257];
  // passes 2 and 3: per key byte (high, or low inside the chosen high byte),
  // 16 lane columns (lanes l and l + 16 share one), so the lanes of a warp do
  // not pile onto one bin's address
  __shared__ float lpm[256 * 16];
  __shared__ float red[kDT / 32];
  __shared__ unsigned ured[kDT / 32];
  const KParams& P = D.P;
  const int tid = threadIdx.x;
  const int i = blockIdx.x;
  if (i >= D.n) return;
  const int row = D.rows[i];
  const bool mine = row >= 0 && row < P.B && full_row(P.temperature, P.top_k, P.vocab_total, row);
  const float* gi = D.gin ? D.gin + static_cast<long long>(kState) * i : nullptr;
  if (!mine || (D.pass > 1 && gi[kSFlag] != 0.f) || (D.pass == 4 && gi[kSHb] == kOwnerKnown)) {   // neutral outputs
    if (tid == 0) {
      if (D.pass == 1) {
        float* o = D.gout + 3ll * i;
        o[0] = -INFINITY; o[1] = __int_as_float(-1); o[2] = 0.f;
      } else if (D.pass == 4) {
        D.gout[i] = 0.f;
      } else if (D.pass == 5) {
        reinterpret_cast<int*>(D.gout)[i] = -1;
      }
    }
    if (D.pass == 2 || D.pass == 3) {
      const int width = (D.pass == 2) ? 256 : 257;
      for (int b = tid; b < width; b += kDT) D.gout[static_cast<long long>(i) * width + b] = 0.f;
    }
    return;
  }
  const float T = P.temperature[row];
  const float rT = __frcp_rn(T);
  const int V = P.V;
  const float M = gi ? gi[kSM] : 0.f;

  if (D.pass == 1) {
    // thread-local running (max z, its lowest id, mass relative to it)
    float zt = -INFINITY, acc = 0.f;
    unsigned kt = 0u, idt = 0xFFFFFFFFu;
    bool nan = false;
    stream_slice<DT>(P, rawb, row, V, [&](const uint16_t* raw, int c0, int len) {
#pragma unroll 4
      for (int j = 0; j < kDPer; ++j) {
        const int e = j * kDT + tid;   // consecutive threads, consecutive entries
        if (e >= len) continue;
        const uint32_t key = key16(raw[e]);
        const float y = Dt::to_f32(raw[e]);
        if (y != y) { nan = true; continue; }
        if (key > kt) { kt = key; idt = static_cast<unsigned>(P.vocab_offset + c0 + e); }
        const float z = quot_rn(y, T, rT);   // the quotient every mass here uses
        if (z == -INFINITY) continue;   // mass 0
        if (z > zt) {
          acc = (zt == -INFINITY) ? 0.f : __fmul_rn(acc, ex2_approx(__fmul_rn(__fsub_rn(zt, z), kLog2e)));
          zt = z;
        }
        acc += ex2_approx(__fmul_rn(__fsub_rn(z, zt), kLog2e));
      }
      return true;
    });
    // block max key, lowest id among its holders, mass rescaled to the block max z
    unsigned kb = __reduce_max_sync(0xFFFFFFFFu, kt);
    if ((tid & 31) == 0) ured[tid >> 5] = kb;
    __syncthreads();
    kb = 0u;
    for (int w = 0; w < kDT / 32; ++w) kb = max(kb, ured[w]);
    __syncthreads();
    unsigned id = (kt == kb) ? idt : 0xFFFFFFFFu;
    id = __reduce_min_sync(0xFFFFFFFFu, id);
    if ((tid & 31) == 0) ured[tid >> 5] = id;
    __syncthreads();
    id = 0xFFFFFFFFu;
    for (int w = 0; w < kDT / 32; ++w) id = min(id, ured[w]);
    const float zmax = __fdiv_rn(C::value(kb), T);
    const float mine = (acc > 0.f) ? __fmul_rn(acc, ex2_approx(__fmul_rn(__fsub_rn(zt, zmax), kLog2e))) : 0.f;
    const float S = bsum(mine, red);
    const int anynan = __syncthreads_or(nan);
    if (tid == 0) {
      float* o = D.gout + 3ll * i;
      o[0] = zmax;
      o[1] = __int_as_float(static_cast<int>(id));
      o[2] = anynan ? __int_as_float(0x7FC00000) : S;   // a NaN logit: the row is refused
    }
    return;
  }

  if (D.pass == 2 || D.pass == 3) {
    const int hb = static_cast<int>(gi[kSHb]);
    if (hb < 0) {   // no top-p on this row: nothing to count
      const int width = (D.pass == 2) ? 256 : 257;
      for (int b = tid; b < width; b += kDT) D.gout[static_cast<long long>(i) * width + b] = 0.f;
      return;
    }
    for (int b = tid; b < 257; b += kDT) hist[b] = 0.f;
    for (int b = tid; b < 256 * 16; b += kDT) lpm[b] = 0.f;
    float above = 0.f;
    __syncthreads();
    stream_slice<DT>(P, rawb, row, V, [&](const uint16_t* raw, int, int len) {
#pragma unroll 4
      for (int j = 0; j < kDPer; ++j) {
        const int e = j * kDT + tid;
        if (e >= len) continue;
        const uint32_t key = key16(raw[e]);
        const int kh = static_cast<int>(key >> 8);
        if (D.pass == 3 && kh < hb) continue;
        const float ms = mass_of(Dt::to_f32(raw[e]), T, rT, M);
        if (!(ms > 0.f)) continue;
        if (D.pass == 2) atomicAdd(&lpm[(kh << 4) | (tid & 15)], ms);
        else if (kh == hb) atomicAdd(&lpm[((key & 255u) << 4) | (tid & 15)], ms);
        else above += ms;
      }
      return true;
    });
    if (D.pass == 3) {
      const float a = bsum(above, red);
      if (tid == 0) hist[256] = a;
    }
    // the lane columns of each bin, in column order
    for (int b = tid; b < 256; b += kDT) {
      float t = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) t += lpm[(b << 4) | c];
      hist[b] = t;
    }
    __syncthreads();
    const int width = (D.pass == 2) ? 256 : 257;
    for (int b = tid; b < width; b += kDT) D.gout[static_cast<long long>(i) * width + b] = hist[b];
    return;
  }

  // passes 4 and 5: the kept keys
  const uint32_t tau = static_cast<uint32_t>(gi[kSTau]);
  const uint32_t kdraw = max(tau ? tie_floor<DT, 16>(tau, T) : 0u, zero_mass_cut<DT, 16>(M, T));
  if (D.pass == 4) {
    float k = 0.f;
    stream_slice<DT>(P, rawb, row, V, [&](const uint16_t* raw, int, int len) {
      for (int j = 0; j < kDPer; ++j) {
        const int e = j * kDT + tid;
        if (e < len && key16(raw[e]) >= kdraw) k += mass_of(Dt::to_f32(raw[e]), T, rT, M);
      }
      return true;
    });
    const float K = bsum(k, red);
    if (tid == 0) D.gout[i] = K;
    return;
  }

  // pass 5: inverse CDF in vocab order over this slice, for the owning rank
  const float t = gi[kST];
  int* out = reinterpret_cast<int*>(D.gout) + i;
  if (!(t >= 0.f)) {
    if (tid == 0) *out = -1;
    return;
  }
  float run = 0.f;       // kept mass of the chunks before this one
  int found = -1, lastk = -1;
  stream_slice<DT>(P, rawb, row, V, [&](const uint16_t* raw, int c0, int len) {
    float s = 0.f;
    int lk = -1;
    for (int j = 0; j < kDPer; ++j) {
      const int e = tid * kDPer + j;
      if (e < len && key16(raw[e]) >= kdraw) {
        const float ms = mass_of(Dt::to_f32(raw[e]), T, rT, M);
        if (ms > 0.f) { s += ms; lk = e; }
      }
    }
    // exclusive prefix of the threads' sums (thread order = vocab order)
    float incl = s;
    const int lane = tid & 31, w = tid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    __syncthreads();
    if (lane == 31) red[w] = incl;
    __syncthreads();
    float wbase = 0.f, total = 0.f;
    for (int q = 0; q < kDT / 32; ++q) {
      if (q < w) wbase += red[q];
      total += red[q];
    }
    const float ex = run + wbase + (incl - s);
    int mine = INT_MAX;
    if (s > 0.f && ex + s > t) {
      float r = ex;
      for (int j = 0; j < kDPer && mine == INT_MAX; ++j) {
        const int e = tid * kDPer + j;
        if (e < len && key16(raw[e]) >= kdraw) {
          const float ms = mass_of(Dt::to_f32(raw[e]), T, rT, M);
          if (ms > 0.f) { r += ms; if (r > t) mine = e; }
        }
      }
      if (mine == INT_MAX) mine = lk;   // reached only after rounding inside this thread
    }
    unsigned m = __reduce_min_sync(0xFFFFFFFFu, static_cast<unsigned>(mine));
    unsigned l = __reduce_max_sync(0xFFFFFFFFu, static_cast<unsigned>(lk + 1));
    __syncthreads();
    if (lane == 0) { ured[w] = m; red[w] = __uint_as_float(l); }
    __syncthreads();
    unsigned mm = 0xFFFFFFFFu, ll = 0u;
    for (int q = 0; q < kDT / 32; ++q) { mm = min(mm, ured[q]); ll = max(ll, __float_as_uint(red[q])); }
    if (mm != static_cast<unsigned>(INT_MAX) && mm != 0xFFFFFFFFu) found = P.vocab_offset + c0 + static_cast<int>(mm);
    else if (ll > 0u) lastk = P.vocab_offset + c0 + static_cast<int>(ll) - 1;
    run += total;
    return found < 0;
  });
  if (tid == 0) *out = found >= 0 ? found : lastk;   // rounding: the slice's last kept entry
}

// ------------------------------------------------------------- combine steps
struct CParams {
  const float* temperature;
  const int* top_k;
  const float* top_p;
  const float* uniforms;                 // [B] or null: Philox from philox_state
  const uint64_t* philox_state;
  int* out;                              // [B] ids (after pass 5)
  int B, vocab, world, rank, pass;
  const int* rows;
  int n;
  const float* G;                        // the combined outputs of pass `pass`
  float* S;                              // [n, kState] row state
};

// The rank whose slice holds the draw: the first with kept mass whose
// inclusive running total (rank order = vocab order) exceeds t = u * sum,
// else (rounding) the last with kept mass.  Writes this rank's local target
// (t minus the ranks before it) or -1; a row without kept mass is refused.
template <class F>
__device__ void pick_owner(float* st, F mass, int world, float u, int rank) {
  float zk = 0.f;
  for (int g = 0; g < world; ++g) zk += mass(g);
  if (!(zk > 0.f)) {
    st[kSFlag] = 2.f;
    return;
  }
  const float t = __fmul_rn(u, zk);
  float cum = 0.f, cum_last = 0.f;
  int owner = -1, last = -1;
  for (int g = 0; g < world; ++g) {
    const float m = mass(g);
    if (m > 0.f) {
      last = g;
      cum_last = cum;
      if (cum + m > t) { owner = g; break; }
    }
    cum += m;
  }
  if (owner < 0) { owner = last; cum = cum_last; }
  st[kST] = (owner == rank) ? fmaxf(__fsub_rn(t, cum), 0.f) : -1.f;
}

__device__ __forceinline__ float draw_uniform(const CParams& C, int row) {
  return C.uniforms ? C.uniforms[row]
                    : row_uniform(C.philox_state[0], C.philox_state[1], static_cast<uint64_t>(row));
}

// One warp per listed row: the combined outputs of pass C.pass (pass 1 and 4:
// all-gathered [world, n, ...] in rank order; passes 2 and 3: summed over the
// ranks; pass 5: the max over the ranks) into the state of the next pass.
__global__ void __launch_bounds__(32) vp_dist_combine_kernel(const __grid_constant__ CParams C) {
  const int i = blockIdx.x;
  const int lane = threadIdx.x;
  if (i >= C.n) return;
  float* st = C.S + static_cast<long long>(kState) * i;
  const int row = C.rows[i];
  const bool mine = row >= 0 && row < C.B && full_row(C.temperature, C.top_k, C.vocab, row);
  if (C.pass == 1) {
    if (!mine) {
      if (lane == 0) st[kSFlag] = 1.f;
      return;
    }
    // M = the row's max z over the ranks
    float M = -INFINITY;
    bool nan = false;
    for (int g = lane; g < C.world; g += 32) {
      const float* o = C.G + 3ll * (static_cast<long long>(g) * C.n + i);
      M = fmaxf(M, o[0]);
      nan |= (o[2] != o[2]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    nan = __any_sync(0xFFFFFFFFu, nan);
    if (lane == 0) {
      const float pp = C.top_p[row];
      const bool topp = pp > 0.f && pp < 1.f;
      const bool bad = nan || !isfinite(M);
      st[kSM] = M;
      st[kSHb] = topp ? 0.f : -1.f;
      st[kSTau] = 0.f;
      st[kST] = -1.f;
      st[kSTarget] = 0.f;
      st[kSFlag] = bad ? 2.f : 0.f;
      if (!topp && !bad) {
        // every entry above the zero-mass cut is kept: each slice's kept mass
        // is its pass-1 mass rescaled to M, so the owner is known now
        pick_owner(st, [&](int g) {
          const float* o = C.G + 3ll * (static_cast<long long>(g) * C.n + i);
          return (o[2] > 0.f) ? __fmul_rn(o[2], ex2_approx(__fmul_rn(__fsub_rn(o[0], M), kLog2e))) : 0.f;
        }, C.world, draw_uniform(C, row), C.rank);
        st[kSHb] = kOwnerKnown;
      }
    }
    return;
  }
  if (!mine) return;
  const float flag = st[kSFlag];
  if (C.pass == 5) {   // the drawn id, on every rank
    if (lane == 0 && flag != 1.f) C.out[row] = (flag == 0.f) ? reinterpret_cast<const int*>(C.G)[i] : -1;
    return;
  }
  if (flag != 0.f) return;
  if (C.pass == 2 || C.pass == 3) {
    if (st[kSHb] < 0.f) return;                   // no top-p
    const float* h = C.G + static_cast<long long>(i) * (C.pass == 2 ? 256 : 257);
    float target;
    if (C.pass == 2) {
      float z = 0.f;
      for (int b = lane; b < 256; b += 32) z += h[b];
      z = warp_sum(z);
      target = __fmul_rn(C.top_p[row], z);
      if (!(z > 0.f)) {
        if (lane == 0) st[kSFlag] = 2.f;
        return;
      }
    } else {
      target = __fsub_rn(st[kSTarget], h[256]);  // past the mass above the high byte
    }
    int bin;
    float above;
    warp_select_seq<float, 256, true>(h, target, &bin, &above);   // lane 0 writes
    if (lane == 0) {
      if (C.pass == 2) {
        st[kSHb] = static_cast<float>(bin);
        st[kSTarget] = target;
      } else {
        st[kSTau] = static_cast<float>(static_cast<int>(st[kSHb]) * 256 + bin);
      }
    }
    return;
  }
  // pass 4: which rank owns the draw, and its local target
  if (lane == 0 && st[kSHb] != kOwnerKnown)
    pick_owner(st, [&](int g) { return C.G[static_cast<long long>(g) * C.n + i]; }, C.world, draw_uniform(C, row),
               C.rank);
}

}  // namespace vd
}  // namespace ecah
