// Fused token-sampler kernel for sm_100a (one thread-block cluster per row).
//
// Each CTA of a row's cluster owns a contiguous vocabulary chunk and keeps it
// resident in shared memory as order-preserving keys of the penalised logit
// y' (16-bit keys while y' stays in the fp16/bf16 model dtype, 32-bit keys
// otherwise).  The logits are read from HBM once; later passes read the
// resident keys 16 bytes at a time and skip whole vectors with one compare
// when no key in them can matter.  CTAs exchange only small summaries (row
// max, histograms, masses) through distributed shared memory, with one
// cluster barrier per exchange.
//
// Op order per row (the reference's): penalty divide -> temperature divide
// (ecahlang/main.py:169-170) -> top-k -> softmax -> top-p -> draw
// (flashinfer top_k_top_p_sampling_from_logits, top_k_first, called at
// ecahlang/main.py:377-379).
//
// Selection runs on y'-keys: z = y'/T is monotone in y', so the k-th largest
// z is (k-th largest y')/T and a z threshold maps back to the least key whose
// quotient reaches it (key_lower_bound, which also keeps keys that the
// float32 divide makes equal).  Only softmax masses need a per-token quotient.
//
// 16-bit keys, k or p active:
//   pass 1  load, penalty patch, raw->key, row max          | barrier
//   pass 2  512-key window below the max: exact count and mass per key;
//           top-p-only rows also accumulate S exactly and a 128-bin
//           fixed-point mass histogram of all keys             | barrier
//           -> tau_k and (usually) tau_p straight from the window
//   pass 3  (nucleus wider than the window) exact masses per key of the
//           selected 512-key bin + exact mass above it          | barrier
//   draw    kept mass per 256-key warp segment, CTA totals      | barrier
//           -> the CTA holding u*Z locates the token by segment, lane, key
// Anything else (32-bit keys, k larger than the window, ties that straddle
// the window) runs the generic radix path: 7|9(|8|8)-bit levels, counts for
// top-k, masses for top-p (fixed-point level 0, exact float sub-bins and an
// exact "mass above" at each deeper level), one barrier per level.
#pragma once

#include <cooperative_groups.h>

#include <climits>

#include "common.cuh"

namespace ecah {

namespace cg = cooperative_groups;

struct KParams {
  const void* logits;
  long long row_stride;
  const int* row_index;    // [B] logits row of each row (NULL: row r)
  int logit_rows;          // rows of the logits buffer (with row_index)
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
  // row kernel and probability kernel: 8192-entry chunks per row, and the
  // finished-row data the probability kernel reads
  int NC;
  void* ws_fin;            // [B] RowFin
  int CL;                  // CTAs per row (cluster size)
  int CH;                  // vocab entries per CTA (multiple of 8)
  int vec_ok;              // 16-byte aligned rows
  float fx_scale;          // fixed-point scale of level-0 masses (2^s)
  float fx_inv;            // 2^-s
  // row kernel (row_kernel.cuh) with a row split over several CTAs
  int parts;                        // CTAs per row, >= 1
  unsigned* part_arrive;            // [B] parts of the row done so far (left 0)
  void* part_hdr;                   // [B, parts] per-part results
  unsigned long long* part_cand;    // [B, parts, kCB] candidates: key << 32 | row index
  float2* part_seg;                 // [B, 32 rounds x 32 warps] segment (mass, reference)
  // vocabulary-parallel local step on the row kernel: V is the slice length
  int vocab_offset;                 // global id of the slice's first entry (0 otherwise)
  int vocab_total;                  // the whole vocabulary
  int cand_cap;                     // list entries per row
  unsigned long long* vp_cand;      // [B, cand_cap] key << 32 | global id, vocab order
  int* vp_count;                    // [B] entries at or above the k-th largest key
  // fused vocabulary-parallel step (lists written straight into every rank's
  // exchange buffer, then a per-row flag; see vp_kernel.cuh)
  void* const* vp_base;             // [vp_world] every rank's exchange buffer, mapped here
  int vp_world, vp_rank, vp_maxb;   // ranks, this rank, rows the buffers hold
  long long vp_lflag, vp_lcount, vp_lcand;   // region offsets in an exchange buffer
  unsigned long long vp_timeout_ns; // per wait on another rank's flag
};

// Element offset of row `row`'s logits: row_index[row] (clamped into
// [0, logit_rows)) rows in when the launch gathers rows, else `row` rows.
__device__ __forceinline__ long long logits_row_offset(const KParams& P, int row) {
  long long r = row;
  if (P.row_index) r = min(max(P.row_index[row], 0), P.logit_rows - 1);
  return r * P.row_stride;
}

// One history entry's penalty applied to a model-dtype value x: the
// repetition divide y = D(x / m), then, with ECAH_FLAG_FREQ_PRES, the additive
// term a = f32(f32(f c) + pi) as y' = D(y - a) -- the penalised logit stays
// in the model dtype, as the reference's `logits / mask_penalty` leaves it.
template <int DT>
__device__ __forceinline__ float penalise(float x, float m, float a) {
  const float y = DType<DT>::round(__fdiv_rn(x, m));
  return (a != 0.f) ? DType<DT>::round(__fsub_rn(y, a)) : y;
}

// The additive term of a history entry seen c > 0 times (0 without
// ECAH_FLAG_FREQ_PRES): f32(f32(f c) + pi).
__device__ __forceinline__ float additive_term(const KParams& P, int row, int c) {
  if (!(P.flags & ECAH_FLAG_FREQ_PRES)) return 0.f;
  const float f = P.freq_pen ? P.freq_pen[row] : 0.f;
  const float pi = P.pres_pen ? P.pres_pen[row] : 0.f;
  return __fadd_rn(__fmul_rn(f, static_cast<float>(c)), pi);
}


constexpr int kNB0 = 128;     // level-0 bins (7-bit digit), lane-private
constexpr int kNBL = 512;     // bins of deeper levels / the key window
constexpr int kWin = 512;     // keys in the window below the row max
constexpr int kMaxSeg = 256;  // warp segments per CTA
constexpr int kMaxCLs = 16;   // CTAs per cluster, at most

// digit layout: 16-bit keys 7|9, 32-bit keys 7|9|8|8 (high to low)
template <int KB> struct Radix;
template <> struct Radix<16> {
  static constexpr int kLevels = 2;
  static __device__ __forceinline__ int shift(int l) { return l == 0 ? 9 : 0; }
  static __device__ __forceinline__ int width(int l) { return l == 0 ? 7 : 9; }
};
template <> struct Radix<32> {
  static constexpr int kLevels = 4;
  static __device__ __forceinline__ int shift(int l) { return l == 0 ? 25 : (l == 1 ? 16 : (l == 2 ? 8 : 0)); }
  static __device__ __forceinline__ int width(int l) { return l == 0 ? 7 : (l == 1 ? 9 : 8); }
};

// 16 bytes of resident keys
template <int KB> struct KV;
template <> struct KV<16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void unpack(const uint4& q, uint32_t (&k)[8]) {
    k[0] = q.x & 0xFFFFu; k[1] = q.x >> 16; k[2] = q.y & 0xFFFFu; k[3] = q.y >> 16;
    k[4] = q.z & 0xFFFFu; k[5] = q.z >> 16; k[6] = q.w & 0xFFFFu; k[7] = q.w >> 16;
  }
  static __device__ __forceinline__ uint32_t vmax(const uint4& q) {
    const uint32_t m = __vmaxu2(__vmaxu2(q.x, q.y), __vmaxu2(q.z, q.w));
    return max(m & 0xFFFFu, m >> 16);
  }
};
template <> struct KV<32> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void unpack(const uint4& q, uint32_t (&k)[4]) {
    k[0] = q.x; k[1] = q.y; k[2] = q.z; k[3] = q.w;
  }
  static __device__ __forceinline__ uint32_t vmax(const uint4& q) { return max(max(q.x, q.y), max(q.z, q.w)); }
};

// Generic-path values published to the cluster, double-buffered by phase
// parity: a set written before barrier s is read by peers between barriers s
// and s+1 and rewritten only after barrier s+1.
struct PubSet {
  unsigned c[kNBL];             // counts of one radix level
  float m[kNBL];                // exact float masses of one radix level
  unsigned long long l0[kNB0];  // level-0 histogram (counts or fixed-point masses)
  float s;                      // exact mass partial (S or "mass above")
};

struct Smem {
  union {
    unsigned lp[kNB0 * 32];     // lane-private level-0 histogram, [bin][lane]
    struct {                    // merged data, after the first barrier
      unsigned cnt[kWin];       // window counts, bin b = key kmax - b
      float e[kWin];            // mass of one token of key kmax - b
      float m[kWin];            // cnt * e
      float l0[kNB0];           // level-0 masses (rescaled to M)
      float e3[kNBL];           // pass 3: mass of one token of key (b0 << 9) | d
    } g;
    struct {                    // generic path
      unsigned mc[kNBL];
      float mm[kNBL];
    } q;
  } u;
  // published to the cluster
  unsigned win[kWin];           // local window counts, bin b = key lmax - b
  unsigned long long l0[kNB0];  // local level-0 fixed-point masses, relative to mref
  unsigned c3[kNBL];            // pass 3: counts of keys in bin b0, index key & 511
  PubSet set[2];
  unsigned lmax;                // CTA-local max key
  float mref;                   // value(lmax) / T
  float sref;                   // sum of exp(z - mref) over the chunk (dense rows)
  float total;                  // kept mass of the CTA (relative to M)
  int first_idx;                // argmax index (greedy)
  // cluster-gathered scalars (local copies)
  unsigned plmax[kMaxCLs];
  float pscale[kMaxCLs];        // exp(mref_c - M)
  float seg[kMaxSeg];           // kept mass per warp segment (draw)
  float red[kThreads / 32];
  int ib[8];
  float fb[8];
};

// Smallest key k in [0, hi] whose quotient value(k)/T reaches zthr.  The
// predicate is monotone on [0, hi] (NaN keys sit below -inf, hi is never a NaN
// key) and callers guarantee it holds at hi.  Starts from a guess key and
// gallops before bisecting.
template <int DT, int KB>
__device__ uint32_t key_lower_bound(float zthr, float T, uint32_t hi) {
  using C = Codec<DT, KB>;
  auto pred = [&](uint32_t k) { return __fdiv_rn(C::value(k), T) >= zthr; };
  if (!pred(hi)) return hi;
  uint32_t lo = 0u, h = hi;  // answer in [lo, h]; pred(h) holds
  const float gv = __fmul_rn(zthr, T);
  uint32_t g;
  if (gv != gv) g = 0u;
  else if (KB == 16) g = C::from_val(DType<DT>::round(gv));
  else g = key32(gv);
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
  while (lo < h) {
    const uint32_t mid = lo + ((h - lo) >> 1);
    if (pred(mid)) h = mid; else lo = mid + 1u;
  }
  return lo;
}

// Least key tying with `key` under the divide: one extra quotient in the
// common no-tie case.
template <int DT, int KB>
__device__ __forceinline__ uint32_t tie_floor(uint32_t key, float T) {
  using C = Codec<DT, KB>;
  if (key == 0u) return 0u;
  const float z = __fdiv_rn(C::value(key), T);
  if (__fdiv_rn(C::value(key - 1u), T) < z) return key;
  return key_lower_bound<DT, KB>(z, T, key);
}

// Warp-level: over positions j = 0..NB-1 (bin = DESC ? NB-1-j : j), find the
// first position whose running total reaches `target`.  Returns the bin and
// the total before it.  If rounding leaves the target unreached, the last
// position with a non-zero value is taken (the most inclusive choice).
template <typename T, int NB, bool DESC>
__device__ void warp_select(const T* hist, T target, int* out_bin, T* out_above) {
  constexpr int PER = NB / 32;
  const int lane = threadIdx.x & 31;
  T v[PER];
  T s = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int pos = lane * PER + j;
    v[j] = hist[DESC ? NB - 1 - pos : pos];
    s += v[j];
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
      T acc = excl;
      int last_nz = -1;
      T acc_last = 0;
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        if (pos < 0) {
          if (v[j] > 0) { last_nz = j; acc_last = acc; }
          if (v[j] > 0 && acc + v[j] >= target) { pos = lane * PER + j; above = acc; }
          acc += v[j];
        }
      }
      if (pos < 0) { pos = lane * PER + (last_nz >= 0 ? last_nz : PER - 1); above = acc_last; }
    }
  } else {
    const unsigned nz = __ballot_sync(0xFFFFFFFFu, s > 0);
    L = nz ? 31 - __clz(nz) : 31;
    if (lane == L) {
      // last non-zero position of this lane and the total before it
      int jb = PER - 1;
      T acc = excl, acc_jb = excl;
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        if (v[j] > 0) { jb = j; acc_jb = acc; }
        acc += v[j];
      }
      pos = lane * PER + jb;
      above = acc_jb;
    }
  }
  pos = __shfl_sync(0xFFFFFFFFu, pos, L);
  above = __shfl_sync(0xFFFFFFFFu, above, L);
  if (lane == 0) { *out_bin = DESC ? NB - 1 - pos : pos; *out_above = above; }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

constexpr int kMaxCL = 16;

// Sum of one value over the CTAs of the cluster, in rank order.  All peer
// loads are issued before the first add so their latency overlaps.
template <typename T>
__device__ __forceinline__ T cluster_sum(const cg::cluster_group& cl, const T* local, int CL) {
  T s = T(0);
  for (int base = 0; base < CL; base += 8) {
    T v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = *cl.map_shared_rank(local, base + j < CL ? base + j : base);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (base + j < CL) s += v[j];
  }
  return s;
}

// Sum of one float per thread in a fixed order (deterministic).
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) t += red[w];
  return t;
}

// Unnormalised softmax mass exp(y/T - M).  The quotient uses Markstein's
// correction step (reciprocal r = RN(1/T), q = RN(y*r), q' = RN(q + r*RN(y - qT)))
// which reproduces the IEEE quotient for every fp16 input (checked exhaustively
// on the B200; it can differ in the sign of a zero or in the last bit of
// sub-1e-30 quotients, neither of which changes the mass).
__device__ __forceinline__ float mass_of(float y, float T, float r, float M) {
  const float q = __fmul_rn(y, r);
  const float z = __fmaf_rn(__fmaf_rn(-q, T, y), r, q);
  return ex2_approx(__fmul_rn(__fsub_rn(z, M), kLog2e));
}

__device__ __forceinline__ unsigned to_fixed(float e, float scale) {
  // round(e * scale) for e * scale < 2^23, read from the low mantissa bits
  return __float_as_uint(__fmaf_rn(e, scale, 8388608.0f)) & 0x7FFFFFu;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Lower bound key below which every token has softmax mass exactly 0 relative
// to m: y < (m - 100 - |m| 2^-20) T gives y/T - m < -99.9 even after the
// roundings of the divide, and ex2 of less than -144 flushes to zero.
template <int DT, int KB>
__device__ __forceinline__ uint32_t zero_mass_cut(float m, float T) {
  const float yc = __fmul_rn(__fsub_rn(__fsub_rn(m, 100.0f), __fmul_rn(fabsf(m), 9.5367431640625e-07f)), T);
  if (!(yc == yc)) return 0u;
  if (KB == 16) return key16(DType<DT>::to_raw(DType<DT>::round_down(yc)));
  return key32(yc);
}

template <int DT, int KB>
__global__ void __launch_bounds__(kThreads, 3) sample_kernel(const KParams P) {
  using Dt = DType<DT>;
  using C = Codec<DT, KB>;
  using Key = typename C::Key;
  using Raw = typename Dt::Raw;
  using R = Radix<KB>;
  constexpr int N = KV<KB>::N;                        // keys per 16-byte vector
  constexpr int VIN = Dt::kVec;                       // logits per 16-byte global load
  constexpr bool kRawInSmem = sizeof(Raw) == sizeof(Key);
  constexpr int kSegPerLane = kMaxSeg / 32;

  extern __shared__ __align__(16) unsigned char dsm[];
  Key* keys = reinterpret_cast<Key*>(dsm);
  uint4* kv4 = reinterpret_cast<uint4*>(dsm);
  __shared__ Smem S;

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int row = blockIdx.x / P.CL;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = rank * P.CH;
  const int n = max(0, min(P.CH, P.V - c0));
  const int nvec = (n + N - 1) / N;
  const Raw* src = reinterpret_cast<const Raw*>(P.logits) + logits_row_offset(P, row) + c0;

  for (int i = tid; i < kWin; i += kThreads) S.win[i] = 0u;
  for (int i = tid; i < kNBL; i += kThreads) S.c3[i] = 0u;
  for (int i = tid; i < kNB0; i += kThreads) S.l0[i] = 0ull;
  if (tid == 0) S.sref = 0.f;
  for (int i = tid; i < kNB0 * 32; i += kThreads) S.u.lp[i] = 0u;
  {
    unsigned* z = reinterpret_cast<unsigned*>(&S.set[0]);
    for (int i = tid; i < static_cast<int>(2 * sizeof(PubSet) / 4); i += kThreads) z[i] = 0u;
  }

  // ------------------------------------------------------------ 1. load
  // Raw logits land in shared memory (converted to keys in pass 1); the tail
  // of the last vector is filled with the minimum key.
  {
    const int nin = (n + VIN - 1) / VIN;
    const int nfull = n / VIN;
    if constexpr (kRawInSmem) {
      if (P.vec_ok) {
        // every 16-byte piece of the chunk in flight at once, no registers held
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        for (int v = tid; v < nfull; v += kThreads) cp_async16(kv4 + v, s4 + v);
        for (int i = nfull * VIN + tid; i < nin * VIN; i += kThreads)
          keys[i] = static_cast<Key>(i < n ? src[i] : (sizeof(Raw) == 2 ? 0xFFFFu : 0xFFFFFFFFu));
      } else {
        for (int i = tid; i < nin * VIN; i += kThreads)
          keys[i] = static_cast<Key>(i < n ? src[i] : (sizeof(Raw) == 2 ? 0xFFFFu : 0xFFFFFFFFu));
      }
    } else {
      // 16-bit logits into 32-bit keys (additive penalties make y' float32)
      if (P.vec_ok) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        for (int v = tid; v < nfull; v += kThreads) {
          const uint4 w = __ldg(s4 + v);
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
          uint4 a, b;
          a.x = C::from_raw(ws[0] & 0xFFFFu); a.y = C::from_raw(ws[0] >> 16);
          a.z = C::from_raw(ws[1] & 0xFFFFu); a.w = C::from_raw(ws[1] >> 16);
          b.x = C::from_raw(ws[2] & 0xFFFFu); b.y = C::from_raw(ws[2] >> 16);
          b.z = C::from_raw(ws[3] & 0xFFFFu); b.w = C::from_raw(ws[3] >> 16);
          kv4[2 * v] = a; kv4[2 * v + 1] = b;
        }
        for (int i = nfull * VIN + tid; i < nin * VIN; i += kThreads)
          keys[i] = static_cast<Key>(i < n ? C::from_raw(src[i]) : 0u);
      } else {
        for (int i = tid; i < nin * VIN; i += kThreads)
          keys[i] = static_cast<Key>(i < n ? C::from_raw(src[i]) : 0u);
      }
    }
  }

  cp_async_wait_all();
  const float T = P.temperature[row];
  const int kk = P.top_k[row];
  const int k_eff = (kk <= 0 || kk >= P.V) ? P.V : kk;
  const float pp = P.top_p[row];
  const bool topk = k_eff < P.V;
  const bool topp = (pp > 0.f && pp < 1.f);
  float u;
  if (P.uniforms) {
    u = P.uniforms[row];
  } else {
    u = row_uniform(P.philox_state[0], P.philox_state[1], static_cast<uint64_t>(row));
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
        // the additive term leaves the logit in the model dtype, as the divide does
        if (fp) y = Dt::round(__fsub_rn(y, __fadd_rn(__fmul_rn(fq, static_cast<float>(cnt)), pr)));
        if constexpr (kRawInSmem) keys[li] = static_cast<Key>(Dt::to_raw(y));
        else keys[li] = static_cast<Key>(C::from_val(y));
      }
    }
  }
  __syncthreads();

  // ------------------------------------------ pass 1: keys, local row max
  uint32_t lmax_all;
  {
    uint32_t tmax = 0u;
    int v = tid;
    for (; v + kThreads < nvec; v += 2 * kThreads) {
      uint4 q0 = kv4[v], q1 = kv4[v + kThreads];
      if constexpr (kRawInSmem) {
        if constexpr (KB == 16) {
          q0.x = key16x2(q0.x); q0.y = key16x2(q0.y); q0.z = key16x2(q0.z); q0.w = key16x2(q0.w);
          q1.x = key16x2(q1.x); q1.y = key16x2(q1.y); q1.z = key16x2(q1.z); q1.w = key16x2(q1.w);
        } else {
          q0.x = key32(__uint_as_float(q0.x)); q0.y = key32(__uint_as_float(q0.y));
          q0.z = key32(__uint_as_float(q0.z)); q0.w = key32(__uint_as_float(q0.w));
          q1.x = key32(__uint_as_float(q1.x)); q1.y = key32(__uint_as_float(q1.y));
          q1.z = key32(__uint_as_float(q1.z)); q1.w = key32(__uint_as_float(q1.w));
        }
        kv4[v] = q0;
        kv4[v + kThreads] = q1;
      }
      tmax = max(tmax, max(KV<KB>::vmax(q0), KV<KB>::vmax(q1)));
    }
    if (v < nvec) {
      uint4 q = kv4[v];
      if constexpr (kRawInSmem) {
        if constexpr (KB == 16) {
          q.x = key16x2(q.x); q.y = key16x2(q.y); q.z = key16x2(q.z); q.w = key16x2(q.w);
        } else {
          q.x = key32(__uint_as_float(q.x)); q.y = key32(__uint_as_float(q.y));
          q.z = key32(__uint_as_float(q.z)); q.w = key32(__uint_as_float(q.w));
        }
        kv4[v] = q;
      }
      tmax = max(tmax, KV<KB>::vmax(q));
    }
    tmax = __reduce_max_sync(0xFFFFFFFFu, tmax);
    if (lane == 0) S.red[warp] = __uint_as_float(tmax);
    __syncthreads();
    uint32_t m = 0u;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) m = max(m, __float_as_uint(S.red[w]));
    if (tid == 0) S.lmax = m;
    lmax_all = m;  // every thread computed the same value
  }
  const uint32_t lmax = lmax_all;
  __syncthreads();

  // ------------------- pass 2 (before any exchange; 16-bit keys, T > 0)
  // top-k rows: counts of the 512 keys below the local max.  Rows without
  // top-k: softmax masses relative to the local max mref (exact sum, 128-bin
  // fixed-point histogram) plus the same window counts.  Peers rescale by
  // exp(mref - M) once the row max M is known.
  // Decisions here use only this CTA's data; everything after the first
  // barrier uses cluster-uniform values (kmax and merged histograms) so every
  // CTA takes the same branches and barriers.
  const float rT = __frcp_rn(T);
  const bool local_ok = (KB == 16) && (T > 0.f) && lmax >= static_cast<uint32_t>(kWin);
  float mref = 0.f;
  if (local_ok) {
    const uint32_t lo_w = lmax - (kWin - 1);
    mref = __fdiv_rn(C::value(lmax), T);
    if (topk) {
      for (int v = tid; v < nvec; v += kThreads) {
        const uint4 q = kv4[v];
        if (KV<KB>::vmax(q) < lo_w) continue;
        uint32_t k[N];
        KV<KB>::unpack(q, k);
#pragma unroll
        for (int j = 0; j < N; ++j)
          if (k[j] >= lo_w) atomicAdd(&S.win[lmax - k[j]], 1u);
      }
    } else if (isfinite(mref)) {
      const uint32_t cut = zero_mass_cut<DT, KB>(mref, T);
      const float fxs = P.fx_scale;
      float sacc = 0.f;
      for (int v = tid; v < nvec; v += kThreads) {
        const uint4 q = kv4[v];
        const uint32_t vm = KV<KB>::vmax(q);
        if (vm < cut) continue;
        uint32_t k[N];
        KV<KB>::unpack(q, k);
        float e[N];
#pragma unroll
        for (int j = 0; j < N; ++j) e[j] = (k[j] >= cut) ? mass_of(C::value(k[j]), T, rT, mref) : 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) {
          sacc += e[j];
          atomicAdd(&S.u.lp[((k[j] >> 9) << 5) | lane], to_fixed(e[j], fxs));
        }
        if (vm >= lo_w) {
#pragma unroll
          for (int j = 0; j < N; ++j)
            if (k[j] >= lo_w) atomicAdd(&S.win[lmax - k[j]], 1u);
        }
      }
      const float sb = block_sum(sacc, S.red);
      __syncthreads();
      if (tid < kNB0) {
        unsigned long long acc = 0ull;
#pragma unroll 8
        for (int j = 0; j < 32; ++j) acc += S.u.lp[(tid << 5) | ((j + tid) & 31)];
        S.l0[tid] = acc;
      }
      if (tid == 0) S.sref = sb;
    }
  }
  if (tid == 0) S.mref = mref;

  cluster.sync();  // ---------------------------------------------------- B1
  if (warp == 0) {
    const uint32_t lm = (lane < P.CL) ? cluster.map_shared_rank(&S, lane)->lmax : 0u;
    const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, lm);
    if (lane < kMaxCLs) S.plmax[lane] = lm;
    if (lane == 0) S.ib[7] = static_cast<int>(km);
  }
  __syncthreads();
  const uint32_t kmax = static_cast<uint32_t>(S.ib[7]);
  int ps = 0;  // parity of the next published set (generic path)

  const float ymax = C::value(kmax);
  const float M = __fdiv_rn(ymax, T);
  const bool greedy = !(T > 0.f) || !isfinite(M);
  // cluster-uniform path flags (finite rows have kmax >= key(-inf) > kWin)
  const bool row_fast = (KB == 16) && (T > 0.f) && kmax >= static_cast<uint32_t>(kWin);
  const bool dense = row_fast && !topk;
  int result = -1;

  if (greedy) {
    // ------------------------------------------- argmax, lowest index wins
    int first = INT_MAX;
    for (int v = tid; v < nvec && first == INT_MAX; v += kThreads) {
      const uint4 q = kv4[v];
      if (KV<KB>::vmax(q) != kmax) continue;
      uint32_t k[N];
      KV<KB>::unpack(q, k);
#pragma unroll
      for (int j = 0; j < N; ++j)
        if (first == INT_MAX && k[j] == kmax && v * N + j < n) first = v * N + j;
    }
    first = __reduce_min_sync(0xFFFFFFFFu, first);
    if (lane == 0) S.red[warp] = __int_as_float(first);
    __syncthreads();
    if (tid == 0) {
      int f = INT_MAX;
      for (int w = 0; w < kThreads / 32; ++w) f = min(f, __float_as_int(S.red[w]));
      S.first_idx = (f == INT_MAX) ? INT_MAX : f + c0;
    }
    cluster.sync();
    if (warp == 0) {
      int f = (lane < P.CL) ? cluster.map_shared_rank(&S, lane)->first_idx : INT_MAX;
      f = __reduce_min_sync(0xFFFFFFFFu, f);
      f = (f == INT_MAX) ? 0 : f;
      if (lane == 0) {
        S.ib[0] = f;
        if (rank == 0) result = f;
        if (P.row_stats && rank == 0) {
          float* st = P.row_stats + 4ll * row;
          st[0] = ymax; st[1] = ymax; st[2] = ymax; st[3] = 1.0f;
        }
      }
    }
    __syncthreads();
    cluster_arrive();
    if (P.probs_out) {
      const int g = S.ib[0] - c0;
      float* po = P.probs_out + static_cast<long long>(row) * P.V + c0;
      for (int i = tid; i < n; i += kThreads) po[i] = (i == g) ? 1.0f : 0.0f;
    }
  } else {
    const uint32_t key_cut = zero_mass_cut<DT, KB>(M, T);
    uint32_t key_lo_k = 0u;   // top-k set: key >= key_lo_k
    uint32_t key_lo = 0u;     // final set: key >= key_lo
    // how the CTA kept masses are obtained: 0 window counts, 1 dense sum,
    // 2 level-0 + pass-3 counts, 3 full draw pass
    int tmode = 3;
    uint32_t b0 = 0u;
    bool generic = !row_fast;
    bool topk_done = false;
    const bool have_local = local_ok && (lmax + static_cast<uint32_t>(kWin) > kmax);

    if (row_fast) {
      // ---------------------------------------------- merge the window
      if (warp == 0) {
        float sc = 0.f;
        if (lane < P.CL) {
          const float mr = cluster.map_shared_rank(&S, lane)->mref;
          sc = dense ? ex2_approx(__fmul_rn(__fsub_rn(mr, M), kLog2e)) : 0.f;
        }
        if (lane < kMaxCLs) S.pscale[lane] = sc;
      }
      __syncthreads();
      for (int b = tid; b < kWin; b += kThreads) {
        unsigned cs = 0u;
        for (int base = 0; base < P.CL; base += 8) {
          unsigned vv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int r = base + j < P.CL ? base + j : base;
            const int idx = b - static_cast<int>(kmax - S.plmax[r]);
            vv[j] = *cluster.map_shared_rank(&S.win[idx >= 0 && idx < kWin ? idx : 0], r);
            if (!(idx >= 0 && idx < kWin) || base + j >= P.CL) vv[j] = 0u;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) cs += vv[j];
        }
        const float e = (kmax >= static_cast<uint32_t>(b)) ? mass_of(C::value(kmax - b), T, rT, M) : 0.f;
        S.u.g.cnt[b] = cs;
        S.u.g.e[b] = e;
        S.u.g.m[b] = __fmul_rn(static_cast<float>(cs), e);
      }
      float S_all = 0.f;
      if (dense) {
        if (tid < kNB0) {
          float a = 0.f;
          for (int r = 0; r < P.CL; ++r)
            a += __fmul_rn(static_cast<float>(*cluster.map_shared_rank(&S.l0[tid], r)) * P.fx_inv, S.pscale[r]);
          S.u.g.l0[tid] = a;
        }
        if (warp == 0) {
          const float sr = (lane < P.CL) ? __fmul_rn(cluster.map_shared_rank(&S, lane)->sref, S.pscale[lane]) : 0.f;
          float incl = sr;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += y;
          }
          if (lane == 31) S.fb[5] = incl;
        }
      }
      __syncthreads();
      if (dense) S_all = S.fb[5];

      // ------------------------------------------------------ top-k
      if (topk) {
        if (warp == 0) {
          unsigned tot = 0u;
#pragma unroll
          for (int j = 0; j < kWin / 32; ++j) tot += S.u.g.cnt[lane * (kWin / 32) + j];
          tot = __reduce_add_sync(0xFFFFFFFFu, tot);
          int b; unsigned above;
          warp_select<unsigned, kWin, false>(S.u.g.cnt, static_cast<unsigned>(k_eff), &b, &above);
          if (lane == 0) {
            int bk = (tot >= static_cast<unsigned>(k_eff)) ? b : -1;
            uint32_t klk = 0u;
            if (bk >= 0) klk = tie_floor<DT, KB>(kmax - static_cast<uint32_t>(bk), T);
            S.ib[0] = bk;
            S.ib[1] = static_cast<int>(klk);
          }
        }
        __syncthreads();
        const int bk = S.ib[0];
        if (bk >= 0) {
          key_lo_k = static_cast<uint32_t>(S.ib[1]);
          key_lo = key_lo_k;
          topk_done = true;
          if (key_lo_k + static_cast<uint32_t>(kWin - 1) >= kmax) tmode = 0;  // K inside the window
          else if (topp) generic = true;
        } else {
          generic = true;
        }
      } else {
        tmode = 1;
      }

      // ------------------------------------------------------ top-p
      if (topp && !generic) {
        const int bmax = topk ? static_cast<int>(kmax - key_lo_k) : kWin - 1;
        for (int b = tid; b < kWin; b += kThreads)
          if (b > bmax) S.u.g.m[b] = 0.f;  // outside the top-k set
        __syncthreads();
        if (warp == 0) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < kWin / 32; ++j) {
            const int b = lane * (kWin / 32) + j;
            s += (b <= bmax) ? S.u.g.m[b] : 0.f;
          }
          s = warp_sum(s);
          const float S_K = topk ? s : S_all;
          const float target = __fmul_rn(pp, S_K);
          int b; float above;
          warp_select<float, kWin, false>(S.u.g.m, target, &b, &above);
          if (lane == 0) {
            const bool in_win = s >= target && b <= bmax;
            S.ib[2] = in_win ? b : -1;
            S.fb[0] = target;
            if (in_win) S.ib[3] = static_cast<int>(tie_floor<DT, KB>(kmax - static_cast<uint32_t>(b), T));
          }
        }
        __syncthreads();
        const float target = S.fb[0];
        if (S.ib[2] >= 0) {
          key_lo = static_cast<uint32_t>(S.ib[3]);
          tmode = (key_lo + static_cast<uint32_t>(kWin - 1) >= kmax) ? 0 : 3;
        } else if (!dense) {
          generic = true;
        } else {
          // nucleus wider than the window: level-0 bin, then exact counts of
          // the 512 keys of that bin
          if (warp == 0) {
            int b; float above;
            warp_select<float, kNB0, true>(S.u.g.l0, target, &b, &above);
            if (lane == 0) { S.ib[4] = b; S.fb[1] = above; }
          }
          __syncthreads();
          b0 = static_cast<uint32_t>(S.ib[4]);
          const float above_b0 = S.fb[1];
          const uint32_t lo3 = b0 << 9, hi3 = lo3 | 511u;
          for (int v = tid; v < nvec; v += kThreads) {
            const uint4 q = kv4[v];
            if (KV<KB>::vmax(q) < lo3) continue;
            uint32_t k[N];
            KV<KB>::unpack(q, k);
#pragma unroll
            for (int j = 0; j < N; ++j)
              if (k[j] >= lo3 && k[j] <= hi3) atomicAdd(&S.c3[k[j] & 511u], 1u);
          }
          for (int d = tid; d < kNBL; d += kThreads)
            S.u.g.e3[d] = mass_of(C::value(lo3 | static_cast<uint32_t>(d)), T, rT, M);
          cluster.sync();  // ---------------------------------------------- B2
          float* mm = S.u.g.m;  // reuse: merged pass-3 masses per key
          for (int d = tid; d < kNBL; d += kThreads)
            mm[d] = __fmul_rn(static_cast<float>(cluster_sum(cluster, &S.c3[d], P.CL)), S.u.g.e3[d]);
          __syncthreads();
          if (warp == 0) {
            int d; float ab;
            warp_select<float, kNBL, true>(mm, __fsub_rn(target, above_b0), &d, &ab);
            if (lane == 0) S.ib[5] = static_cast<int>(tie_floor<DT, KB>(lo3 | static_cast<uint32_t>(d), T));
          }
          __syncthreads();
          key_lo = static_cast<uint32_t>(S.ib[5]);
          tmode = (key_lo >= lo3) ? 2 : 3;
        }
      }
    }

    // ------------------------------------------------ generic radix path
    if (generic) {
      tmode = 3;
      if (topk && !topk_done) {
        uint32_t prefix = 0u;
        unsigned krem = static_cast<unsigned>(k_eff);
        for (int lev = 0; lev < R::kLevels; ++lev) {
          const int sh = R::shift(lev), wd = R::width(lev);
          PubSet& Q = S.set[ps & 1];
          if (lev == 0) {
            for (int i = tid; i < kNB0 * 32; i += kThreads) S.u.lp[i] = 0u;
            __syncthreads();
          }
          for (int v = tid; v < nvec; v += kThreads) {
            const uint4 q = kv4[v];
            if (lev > 0 && KV<KB>::vmax(q) < (prefix << (sh + wd))) continue;
            uint32_t k[N];
            KV<KB>::unpack(q, k);
            const int lim = min(N, n - v * N);
#pragma unroll
            for (int j = 0; j < N; ++j) {
              if (j >= lim) break;
              const uint32_t kj = k[j];
              if (lev == 0) {
                atomicAdd(&S.u.lp[((kj >> sh) << 5) | lane], 1u);
              } else if ((kj >> (sh + wd)) == prefix) {
                atomicAdd(&Q.c[(kj >> sh) & ((1u << wd) - 1u)], 1u);
              }
            }
          }
          if (lev == 0) {
            __syncthreads();
            if (tid < kNB0) {
              unsigned long long acc = 0ull;
#pragma unroll 8
              for (int j = 0; j < 32; ++j) acc += S.u.lp[(tid << 5) | ((j + tid) & 31)];
              Q.l0[tid] = acc;
            }
          }
          cluster.sync();
          const int nb = 1 << wd;
          for (int b = tid; b < nb; b += kThreads)
            S.u.q.mc[b] = (lev == 0) ? static_cast<unsigned>(cluster_sum(cluster, &S.set[ps & 1].l0[b], P.CL))
                                     : cluster_sum(cluster, &S.set[ps & 1].c[b], P.CL);
          ++ps;
          {
            unsigned* z = reinterpret_cast<unsigned*>(&S.set[ps & 1]);
            for (int i = tid; i < static_cast<int>(sizeof(PubSet) / 4); i += kThreads) z[i] = 0u;
          }
          __syncthreads();
          if (warp == 0) {
            int b; unsigned above;
            if (nb == 128) warp_select<unsigned, 128, true>(S.u.q.mc, krem, &b, &above);
            else if (nb == 256) warp_select<unsigned, 256, true>(S.u.q.mc, krem, &b, &above);
            else warp_select<unsigned, 512, true>(S.u.q.mc, krem, &b, &above);
            if (lane == 0) { S.ib[0] = b; S.ib[1] = static_cast<int>(above); }
          }
          __syncthreads();
          prefix = (prefix << wd) | static_cast<uint32_t>(S.ib[0]);
          krem -= static_cast<unsigned>(S.ib[1]);
          __syncthreads();
        }
        key_lo_k = tie_floor<DT, KB>(prefix, T);
      }
      key_lo = key_lo_k;
      if (topp) {
        const uint32_t klo = max(key_lo_k, key_cut);
        uint32_t prefix = 0u;
        float target = 0.f;
        for (int lev = 0; lev < R::kLevels; ++lev) {
          const int sh = R::shift(lev), wd = R::width(lev);
          PubSet& Q = S.set[ps & 1];
          float acc = 0.f;  // level 0: S_K partial; deeper: mass above the prefix range
          const float fxs = P.fx_scale;
          if (lev == 0) {
            for (int i = tid; i < kNB0 * 32; i += kThreads) S.u.lp[i] = 0u;
            __syncthreads();
          }
          const uint32_t lo_lev = (lev == 0) ? klo : max(klo, prefix << (sh + wd));
          for (int v = tid; v < nvec; v += kThreads) {
            const uint4 q = kv4[v];
            if (KV<KB>::vmax(q) < lo_lev) continue;
            uint32_t k[N];
            KV<KB>::unpack(q, k);
#pragma unroll
            for (int j = 0; j < N; ++j) {
              const uint32_t kj = k[j];
              if (kj < klo) continue;
              if (lev == 0) {
                const float e = mass_of(C::value(kj), T, rT, M);
                acc += e;
                atomicAdd(&S.u.lp[((kj >> sh) << 5) | lane], to_fixed(e, fxs));
              } else {
                const uint32_t hi = kj >> (sh + wd);
                if (hi < prefix) continue;
                const float e = mass_of(C::value(kj), T, rT, M);
                if (hi == prefix) atomicAdd(&Q.m[(kj >> sh) & ((1u << wd) - 1u)], e);
                else acc += e;
              }
            }
          }
          const float accb = block_sum(acc, S.red);
          if (lev == 0) {
            if (tid < kNB0) {
              unsigned long long a2 = 0ull;
#pragma unroll 8
              for (int j = 0; j < 32; ++j) a2 += S.u.lp[(tid << 5) | ((j + tid) & 31)];
              Q.l0[tid] = a2;
            }
          }
          if (tid == 0) Q.s = accb;
          cluster.sync();
          const int nb = 1 << wd;
          for (int b = tid; b < nb; b += kThreads)
            S.u.q.mm[b] = (lev == 0) ? static_cast<float>(cluster_sum(cluster, &S.set[ps & 1].l0[b], P.CL)) * P.fx_inv
                                     : cluster_sum(cluster, &S.set[ps & 1].m[b], P.CL);
          if (tid == 0) S.fb[2] = cluster_sum(cluster, &S.set[ps & 1].s, P.CL);
          ++ps;
          {
            unsigned* z = reinterpret_cast<unsigned*>(&S.set[ps & 1]);
            for (int i = tid; i < static_cast<int>(sizeof(PubSet) / 4); i += kThreads) z[i] = 0u;
          }
          __syncthreads();
          if (lev == 0) target = __fmul_rn(pp, S.fb[2]);
          const float goal = (lev == 0) ? target : __fsub_rn(target, S.fb[2]);
          if (warp == 0) {
            int b; float above;
            if (nb == 128) warp_select<float, 128, true>(S.u.q.mm, goal, &b, &above);
            else if (nb == 256) warp_select<float, 256, true>(S.u.q.mm, goal, &b, &above);
            else warp_select<float, 512, true>(S.u.q.mm, goal, &b, &above);
            if (lane == 0) S.ib[0] = b;
          }
          __syncthreads();
          prefix = (prefix << wd) | static_cast<uint32_t>(S.ib[0]);
          __syncthreads();
        }
        key_lo = max(tie_floor<DT, KB>(prefix, T), key_lo_k);
      }
    }

    // ---------------------------------------------------------- draw
    const uint32_t kdraw = max(key_lo, key_cut);
    const int nseg = (nvec + 31) / 32;
    auto segment_pass = [&]() {
      // kept mass per warp segment (32 consecutive vectors); padding keys are 0
      for (int s = warp; s < nseg; s += kThreads / 32) {
        const int v = s * 32 + lane;
        float acc = 0.f;
        if (v < nvec) {
          const uint4 q = kv4[v];
          if (KV<KB>::vmax(q) >= kdraw) {
            uint32_t k[N];
            KV<KB>::unpack(q, k);
#pragma unroll
            for (int j = 0; j < N; ++j)
              if (k[j] >= kdraw) acc += mass_of(C::value(k[j]), T, rT, M);
          }
        }
        if (__any_sync(0xFFFFFFFFu, acc > 0.f)) acc = warp_sum(acc);
        if (lane == 0) S.seg[s] = acc;
      }
      __syncthreads();
    };
    auto segment_total = [&]() -> float {  // warp 0: lanes own contiguous segment ranges
      float sl = 0.f;
#pragma unroll
      for (int j = 0; j < kSegPerLane; ++j) {
        const int s = lane * kSegPerLane + j;
        if (s < nseg) sl += S.seg[s];
      }
      return sl;
    };
    // kept mass of this CTA
    if (tmode == 3) {
      segment_pass();
      if (warp == 0) {
        float incl = segment_total();
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += y;
        }
        if (lane == 31) S.total = incl;
      }
    } else if (tmode == 1) {
      if (tid == 0) S.total = __fmul_rn(S.sref, S.pscale[rank]);
    } else if (tmode == 0) {
      // this CTA's window keys >= kdraw, at per-key masses of the merged window
      float acc = 0.f;
      if (have_local) {
        const int dl = static_cast<int>(kmax - lmax);
        for (int b = tid; b < kWin; b += kThreads) {
          const uint32_t key = lmax - static_cast<uint32_t>(b);
          const int gb = b + dl;
          if (key >= kdraw && gb < kWin && S.win[b]) acc += __fmul_rn(static_cast<float>(S.win[b]), S.u.g.e[gb]);
        }
      }
      const float t = block_sum(acc, S.red);
      if (tid == 0) S.total = t;
    } else {
      // level-0 bins above b0 (fixed point) + this CTA's pass-3 keys >= key_lo
      float acc = 0.f;
      if (tid < kNB0 && static_cast<uint32_t>(tid) > b0)
        acc = __fmul_rn(static_cast<float>(S.l0[tid]) * P.fx_inv, S.pscale[rank]);
      for (int d = tid; d < kNBL; d += kThreads)
        if (((b0 << 9) | static_cast<uint32_t>(d)) >= kdraw && S.c3[d])
          acc += __fmul_rn(static_cast<float>(S.c3[d]), S.u.g.e3[d]);
      const float t = block_sum(acc, S.red);
      if (tid == 0) S.total = t;
    }
    cluster.sync();  // ------------------------------------------------ draw
    if (warp == 0) {
      // lane r holds CTA r's total; running sums in rank order
      const float tr = (lane < P.CL) ? cluster.map_shared_rank(&S, lane)->total : 0.f;
      float incl = tr;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      const float Z = __shfl_sync(0xFFFFFFFFu, incl, 31);
      float excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
      if (lane == 0) excl = 0.f;
      const float target = __fmul_rn(u, Z);
      const unsigned hit = __ballot_sync(0xFFFFFFFFu, tr > 0.f && incl > target);
      const unsigned nz = __ballot_sync(0xFFFFFFFFu, tr > 0.f);
      int rsel = -1, take_last = 0;
      if (hit) rsel = __ffs(hit) - 1;
      else if (nz) { rsel = 31 - __clz(nz); take_last = 1; }
      const float run_sel = __shfl_sync(0xFFFFFFFFu, excl, rsel < 0 ? 0 : rsel);
      if (lane == 0) {
        S.ib[0] = rsel;
        S.ib[1] = take_last;
        S.fb[0] = __fsub_rn(target, run_sel);
        S.fb[1] = Z;
        if (P.row_stats && rank == 0) {
          float* st = P.row_stats + 4ll * row;
          st[0] = topk ? C::value(key_lo_k) : -INFINITY;
          st[1] = (topk || topp) ? C::value(key_lo) : -INFINITY;
          st[2] = M;
          st[3] = Z;
        }
      }
    }
    __syncthreads();
    cluster_arrive();  // peers may still read this CTA's shared memory until the final wait
    const int rsel = S.ib[0];
    if (rsel == rank) {
      if (tmode != 3) segment_pass();
      if (warp == 0) {
        const bool take_last = S.ib[1] != 0;
        const float rem = S.fb[0];
        // segment: lane ranges, then sequential within the lane
        const float sl = segment_total();
        float incl = sl;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += y;
        }
        float excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
        if (lane == 0) excl = 0.f;
        const unsigned hit = take_last ? 0u : __ballot_sync(0xFFFFFFFFu, sl > 0.f && incl > rem);
        bool last = take_last;
        int L;
        if (hit) {
          L = __ffs(hit) - 1;
        } else {
          const unsigned nz = __ballot_sync(0xFFFFFFFFu, sl > 0.f);
          L = nz ? 31 - __clz(nz) : 0;
          last = true;
        }
        int sel = -1;
        float rem2 = 0.f;
        if (lane == L) {
          float run = excl;
          int slast = -1;
          for (int j = 0; j < kSegPerLane; ++j) {
            const int s = lane * kSegPerLane + j;
            if (s >= nseg) break;
            const float vs = S.seg[s];
            if (vs > 0.f) slast = s;
            if (!last && sel < 0 && vs > 0.f && run + vs > rem) { sel = s; rem2 = __fsub_rn(rem, run); }
            run += vs;
          }
          if (sel < 0) { sel = slast; last = true; }
          if (sel < 0) sel = 0;
        }
        sel = __shfl_sync(0xFFFFFFFFu, sel, L);
        rem2 = __shfl_sync(0xFFFFFFFFu, rem2, L);
        last = __shfl_sync(0xFFFFFFFFu, last, L);
        // within the segment: one vector per lane
        const int v = sel * 32 + lane;
        float ev[N];
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) ev[j] = 0.f;
        if (v < nvec) {
          const uint4 q = kv4[v];
          uint32_t k[N];
          KV<KB>::unpack(q, k);
#pragma unroll
          for (int j = 0; j < N; ++j) {
            if (k[j] >= kdraw) ev[j] = mass_of(C::value(k[j]), T, rT, M);
            acc += ev[j];
          }
        }
        float inc2 = acc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xFFFFFFFFu, inc2, o);
          if (lane >= o) inc2 += y;
        }
        float exc2 = __shfl_up_sync(0xFFFFFFFFu, inc2, 1);
        if (lane == 0) exc2 = 0.f;
        const unsigned hit2 = last ? 0u : __ballot_sync(0xFFFFFFFFu, acc > 0.f && inc2 > rem2);
        int L2;
        if (hit2) {
          L2 = __ffs(hit2) - 1;
        } else {
          const unsigned nz = __ballot_sync(0xFFFFFFFFu, acc > 0.f);
          L2 = nz ? 31 - __clz(nz) : 0;
        }
        if (lane == L2) {
          int pick = -1, lastpos = -1;
          float run = exc2;
#pragma unroll
          for (int j = 0; j < N; ++j) {
            if (ev[j] > 0.f) {
              lastpos = j;
              run += ev[j];
              if (hit2 && pick < 0 && run > rem2) pick = j;
            }
          }
          if (pick < 0) pick = lastpos;
          if (pick < 0) pick = 0;
          result = c0 + v * N + pick;
        }
      }
    }
    if (rsel < 0) {
      // no finite mass anywhere: fall back to the lowest index of the row max
      int first = INT_MAX;
      for (int i = tid; i < n; i += kThreads)
        if (static_cast<uint32_t>(keys[i]) == kmax) { first = i; break; }
      first = __reduce_min_sync(0xFFFFFFFFu, first);
      if (lane == 0) S.red[warp] = __int_as_float(first);
      __syncthreads();
      if (tid == 0) {
        int f = INT_MAX;
        for (int w = 0; w < kThreads / 32; ++w) f = min(f, __float_as_int(S.red[w]));
        S.first_idx = (f == INT_MAX) ? INT_MAX : f + c0;
      }
      cluster_wait();
      cluster.sync();
      if (rank == 0 && warp == 0) {
        int f = (lane < P.CL) ? cluster.map_shared_rank(&S, lane)->first_idx : INT_MAX;
        f = __reduce_min_sync(0xFFFFFFFFu, f);
        if (lane == 0) result = (f == INT_MAX) ? 0 : f;
      }
      cluster_arrive();
    }
    if (P.probs_out) {
      const float Z = S.fb[1];
      float* po = P.probs_out + static_cast<long long>(row) * P.V + c0;
      for (int i = tid; i < n; i += kThreads) {
        const uint32_t k = keys[i];
        po[i] = (k >= kdraw && rsel >= 0) ? __fdiv_rn(mass_of(C::value(k), T, rT, M), Z) : 0.0f;
      }
    }
  }

  if (result >= 0) P.out[row] = min(result, P.V - 1);
  __syncthreads();  // converged warps for the aligned cluster barrier
  cluster_wait();   // every peer is done reading this CTA's shared memory

  if (!P.uniforms && rank == 0 && tid == 0) {
    // the last cluster to finish advances the Philox offset; every cluster
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

}  // namespace ecah
