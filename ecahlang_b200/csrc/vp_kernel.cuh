// Vocab-parallel sampling (fp16/bf16 logits): every rank holds a contiguous
// slice [vocab_offset, vocab_offset + vocab_local) of each row.
//
// The local step is the row kernel's stream over the slice
// (rk::vp_local_row_kernel): repetition-penalty patch of the row's history
// tokens that fall in the slice, the slice's k-th largest key (k = top_k, 1
// for greedy rows) and every slice entry whose key is >= that key -- ties
// included -- in vocab order as (key << 32 | global id), up to cand_cap of
// them, plus their count.
//
// Because the row's k-th largest key is >= every slice's k-th largest key,
// the union of the slices' lists holds every entry of the row's top-k set.
// After an all-gather of the lists, vp_merge_kernel (one CTA per row, the
// same on every rank) takes the row max, the top-k threshold (exact counts
// per key of the merged entries), softmax masses, the top-p threshold and the
// inverse-CDF draw in global vocab order with the row's uniform, so every
// rank returns the same token.  Op order, masses and tie rules are those of
// the other sampler kernels.
//
// The fused step (rk::vp_step_row_kernel) does all of it in one kernel over
// NVLink peer memory.  Every rank owns an exchange buffer that every other
// rank has mapped (CUDA IPC):
//   [0, 256)  header: step epoch (u32 at 0), finished-row counter (u32 at 4),
//             error word (i32 at 8: a wait ran out);
//   flag      [world][maxb] u32: rank g sets flag[g][row] = epoch once its
//             list of the row is in this buffer;
//   count     [2][world][maxb] i32 and cand [2][world][maxb][cap] u64: rank
//             g's counts and lists, double-buffered by epoch parity.
// Per row a CTA streams its slice, stores the list and count into its slot of
// every rank's buffer (plain stores over NVLink, no multicast).  Once all its
// rows are out, the CTA fences at system scope and sets their flags in every
// buffer (st.release.sys), then waits for every rank's flag of each
// row in its own buffer (ld.acquire.sys, bounded by vp_timeout_ns) and
// merges the row from its own buffer.  No CTA waits before it has flagged
// all its rows, so no wait depends on another wait.
// A rank reaches step s + 2 only after every rank has flagged every row of
// step s + 1, which each rank does after finishing step s, so the parity
// buffer a rank reads is never rewritten under it; flags only grow, so a
// flag read late compares >= the epoch.
#pragma once

#include <type_traits>

#include "row_kernel.cuh"

namespace ecah {
namespace vp {

constexpr int kMT = 256;                 // threads of the merge kernel
constexpr int kMW = kMT / 32;
constexpr int kMaxMerged = 2048;         // world * cand_cap entries per row, at most
constexpr int kWin = 4096;               // merge histogram: keys below the row max

// what the merge reads (the local step runs on the row kernel's KParams)
struct VParams {
  int B, V;
  int Bs;                                 // rows between two ranks' lists (B, or the buffers' maxb)
  const float* temperature;
  const int* top_k;
  const float* top_p;
  int cap;                                // candidates per row and rank
  int world;
  const unsigned long long* all_cand;     // [world, Bs, cap]
  const int* all_count;                   // [world, Bs] (> cap: truncated)
  const float* uniforms;
  unsigned long long* philox_state;
  unsigned* done_counter;
  unsigned* epoch;                        // fused step: advanced with the Philox offset
  int* out;
  float* row_stats;
};

// ------------------------------------------------------------ merge step
template <int NT>
struct MSmem {
  unsigned long long c[kMaxMerged];   // merged entries, rank order (= vocab order)
  unsigned cnt[kWin];                 // counts per key, bin b = key kmax - b
  float red[NT / 32];
  unsigned ured[NT / 32];
  int ofs[65];
  int ib[8];
  float fb[8];
};

// A merge runs on a group of NT threads of the CTA (gt: the thread's index in
// the group) that meet at hardware barrier `bar` (0 when the group is the
// whole CTA).
template <int NT>
__device__ __forceinline__ void gsync(int bar) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(NT) : "memory");
}

template <int NT>
__device__ __forceinline__ unsigned mblock_max(unsigned v, unsigned* red, int gt, int bar) {
  v = __reduce_max_sync(0xFFFFFFFFu, v);
  if ((gt & 31) == 0) red[gt >> 5] = v;
  gsync<NT>(bar);
  unsigned m = 0u;
  for (int w = 0; w < NT / 32; ++w) m = max(m, red[w]);
  gsync<NT>(bar);
  return m;
}

template <int NT>
__device__ __forceinline__ unsigned mblock_min(unsigned v, unsigned* red, int gt, int bar) {
  v = __reduce_min_sync(0xFFFFFFFFu, v);
  if ((gt & 31) == 0) red[gt >> 5] = v;
  gsync<NT>(bar);
  unsigned m = 0xFFFFFFFFu;
  for (int w = 0; w < NT / 32; ++w) m = min(m, red[w]);
  gsync<NT>(bar);
  return m;
}

// Over kWin bins in ascending order (thread t: bins t*PB .. t*PB+PB-1), the
// first whose running sum reaches the target -- `target`, or, when frac > 0,
// frac times the bins' sum -- and where rounding leaves it unreached, the
// last non-zero bin; -1 when every bin is zero.  *total = the bins' sum.
// Every thread gets the result.
template <int NT, typename V>
__device__ __forceinline__ int mselect(const V* hist, V target, float frac, MSmem<NT>& S, V* total, int gt, int bar) {
  constexpr int PB = kWin / NT, NW = NT / 32;
  const int tid = gt, lane = tid & 31, warp = tid >> 5;
  V v[PB], s = V(0);
#pragma unroll
  for (int j = 0; j < PB; ++j) { v[j] = hist[tid * PB + j]; s += v[j]; }
  V incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const V y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) reinterpret_cast<V*>(S.red)[warp] = incl;
  gsync<NT>(bar);
  V base = V(0), tot = V(0);
  for (int w = 0; w < NW; ++w) {
    const V x = reinterpret_cast<const V*>(S.red)[w];
    if (w < warp) base += x;
    tot += x;
  }
  *total = tot;
  if constexpr (std::is_same<V, float>::value) {
    if (frac > 0.f) target = __fmul_rn(frac, tot);
  }
  const V ex = base + incl - s;
  int mine = INT_MAX, last = -1;
  V acc = ex;
#pragma unroll
  for (int j = 0; j < PB; ++j) {
    if (v[j] > V(0)) {
      last = tid * PB + j;
      if (mine == INT_MAX && acc + v[j] >= target) mine = tid * PB + j;
    }
    acc += v[j];
  }
  const unsigned pick = mblock_min<NT>(static_cast<unsigned>(mine), S.ured, gt, bar);
  if (pick != static_cast<unsigned>(INT_MAX)) return static_cast<int>(pick);
  return static_cast<int>(mblock_max<NT>(static_cast<unsigned>(last + 1), S.ured, gt, bar)) - 1;
}

// One row of the merge by a group of NT threads (gt, bar: see gsync).
// `lost`: a rank's list never arrived (the fused step's wait ran out); the
// row gets -1.
template <int DT, int NT>
__device__ __forceinline__ void merge_row(const VParams& P, MSmem<NT>& S, int row, bool lost, int gt, int bar) {
  constexpr int NW = NT / 32;
  using C = Codec<DT, 16>;
  const int tid = gt, lane = tid & 31;

  // merged entries of the row: rank by rank (each rank's list is in vocab order)
  if (tid == 0) {
    int acc = 0, bad = 0;
    for (int g = 0; g < P.world; ++g) {
      const int c = lost ? 0 : P.all_count[static_cast<long long>(g) * P.Bs + row];
      if (c > P.cap) bad = 1;
      S.ofs[g] = acc;
      acc += min(c, P.cap);
    }
    S.ofs[P.world] = acc;
    S.ib[0] = bad | (lost ? 1 : 0);
  }
  gsync<NT>(bar);
  const int total = S.ofs[P.world];
  const bool truncated = S.ib[0] != 0;
  for (int g = 0; g < P.world; ++g) {
    const int c = S.ofs[g + 1] - S.ofs[g];
    const unsigned long long* src = P.all_cand + (static_cast<long long>(g) * P.Bs + row) * P.cap;
    for (int i = tid; i < c; i += NT) S.c[S.ofs[g] + i] = src[i];
  }
  gsync<NT>(bar);

  const float T = P.temperature[row];
  const int kk = P.top_k[row];
  const int k_eff = (kk <= 0 || kk >= P.V) ? P.V : kk;
  const float pp = P.top_p[row];
  const bool topk = k_eff < P.V;
  const bool topp = (pp > 0.f && pp < 1.f);

  // row max and its lowest id
  unsigned km = 0u;
  for (int i = tid; i < total; i += NT) km = max(km, static_cast<unsigned>(S.c[i] >> 32));
  const unsigned kmax = mblock_max<NT>(km, S.ured, gt, bar);
  unsigned fid = 0xFFFFFFFFu;
  for (int i = tid; i < total; i += NT)
    if (static_cast<unsigned>(S.c[i] >> 32) == kmax) fid = min(fid, static_cast<unsigned>(S.c[i] & 0xFFFFFFFFu));
  const unsigned first = mblock_min<NT>(fid, S.ured, gt, bar);
  const float ymax = C::value(kmax);
  const float M = __fdiv_rn(ymax, T);
  // a truncated sampled row is refused whatever its lists hold (a rank whose
  // k exceeds cand_cap writes no list); greedy rows need only each rank's
  // first entries, which a truncated list keeps
  const bool greedy = !(T > 0.f) || (!truncated && !isfinite(M));
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
    unsigned* rlo = S.cnt;   // per rank (scratch until the histogram below)
    if (tid < P.world) rlo[tid] = 0xFFFFFFFFu;
    gsync<NT>(bar);
    for (int i = tid, g = 0; i < total; i += NT) {
      while (i >= S.ofs[g + 1]) ++g;
      atomicMin(&rlo[g], static_cast<unsigned>(S.c[i] >> 32));
    }
    gsync<NT>(bar);
    const unsigned fl = (tid < P.world && S.ofs[tid + 1] > S.ofs[tid]) ? rlo[tid] : 0u;
    uint32_t F = mblock_max<NT>(fl, S.ured, gt, bar);
    if (kmax >= static_cast<uint32_t>(kWin) && F < kmax - static_cast<uint32_t>(kWin - 1)) F = kmax - static_cast<uint32_t>(kWin - 1);
    for (int b = tid; b < kWin; b += NT) S.cnt[b] = 0u;
    gsync<NT>(bar);
    for (int i = tid; i < total; i += NT) {
      const unsigned key = static_cast<unsigned>(S.c[i] >> 32);
      if (key >= F) atomicAdd(&S.cnt[kmax - key], 1u);
    }
    gsync<NT>(bar);
    if (topk) {
      unsigned tot;
      const int b = mselect<NT, unsigned>(S.cnt, static_cast<unsigned>(k_eff), 0.f, S, &tot, gt, bar);
      ok = tot >= static_cast<unsigned>(k_eff) && b >= 0;
      if (ok) {
        key_lo_k = tie_floor<DT, 16>(kmax - static_cast<uint32_t>(b), T);   // every thread, same value
        ok = key_lo_k >= F;
      }
    } else {
      ok = false;  // without top-k the slices' lists do not hold the row
    }
    key_lo = key_lo_k;
    if (ok && topp) {
      const int bk = static_cast<int>(kmax - key_lo_k);
      float* mb = reinterpret_cast<float*>(S.cnt);
      for (int b = tid; b < kWin; b += NT) {
        const unsigned cn = S.cnt[b];
        mb[b] = (b <= bk && cn) ? __fmul_rn(static_cast<float>(cn), mass_of(C::value(kmax - static_cast<uint32_t>(b)), T, rT, M)) : 0.f;
      }
      gsync<NT>(bar);
      float s;   // the top-k set's mass; the target is pp times it
      const int b = mselect<NT, float>(mb, 0.f, pp, S, &s, gt, bar);
      key_lo = max(tie_floor<DT, 16>(kmax - static_cast<uint32_t>(max(b, 0)), T), key_lo_k);
    }
    if (ok) {
      // inverse CDF over the merged entries in vocab order (thread t: a contiguous stretch)
      const uint32_t kdraw = max(key_lo, key_cut);
      const int per = (total + NT - 1) / NT;
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
      gsync<NT>(bar);
      float base = 0.f, tot = 0.f;
      for (int w = 0; w < NW; ++w) {
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
      gsync<NT>(bar);
      const unsigned pick = mblock_min<NT>(static_cast<unsigned>(mine), S.ured, gt, bar);
      const unsigned last = mblock_max<NT>(static_cast<unsigned>(lastp + 1), S.ured, gt, bar);
      if (pick != static_cast<unsigned>(INT_MAX)) result = static_cast<int>(S.c[pick] & 0xFFFFFFFFu);
      else if (last > 0u) result = static_cast<int>(S.c[last - 1u] & 0xFFFFFFFFu);
      else ok = false;
    }
  }

  if (tid == 0) {
    P.out[row] = (!lost && (greedy || ok)) ? min(result, P.V - 1) : -1;
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
    const bool philox = !P.uniforms && P.philox_state;
    if (philox || P.epoch) {
      // the last row to finish advances the Philox offset and the epoch
      __threadfence();
      const unsigned prev = atomicAdd(P.done_counter, 1u);
      if (prev == static_cast<unsigned>(P.B) - 1u) {
        if (philox) P.philox_state[1] += 1ull;
        if (P.epoch) *P.epoch += 1u;
        *P.done_counter = 0u;
        __threadfence();
      }
    }
  }
}

template <int DT>
__global__ void __launch_bounds__(kMT) vp_merge_kernel(const __grid_constant__ VParams P) {
  __shared__ MSmem<kMT> S;
  merge_row<DT, kMT>(P, S, blockIdx.x, false, threadIdx.x, 0);
}

}  // namespace vp

// ------------------------------------------------------------ fused step
namespace rk {

constexpr unsigned kSpinMax = 1u << 24;   // backstop to the time limit of a wait
static_assert(kMergeGroups * sizeof(vp::MSmem<kMergeT>) <= sizeof(RSmem::stage) + sizeof(RSmem::lp),
              "merge scratch of the fused step must fit in the stages and the histogram scratch");

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

template <int DT>
__device__ __noinline__ void vp_fused_finish(const KParams& P, RSmem& S, int row, unsigned epoch, int g) {
  // group g (threads 256 g .. 256 g + 255, hardware barrier 1 + g) and its
  // own merge scratch, carved from the stages and the histogram scratch
  constexpr int NT = kMergeT;
  const int tid = threadIdx.x - NT * g, bar = 1 + g;
  vp::MSmem<NT>& M_S = reinterpret_cast<vp::MSmem<NT>*>(&S.stage[0][0])[g];
  const int world = P.vp_world;
  char* own = static_cast<char*>(P.vp_base[P.vp_rank]);
  int* err = reinterpret_cast<int*>(own + 8);
  int lost = 0;
  if (tid < world) {
    const unsigned* fl = reinterpret_cast<const unsigned*>(own + P.vp_lflag) + static_cast<long long>(tid) * P.vp_maxb + row;
    if (*static_cast<volatile int*>(err) != 0) {
      lost = 1;   // an earlier wait of this step ran out: wait no more
    } else {
      const unsigned long long t0 = global_ns();
      for (unsigned it = 0;; ++it) {
        if (static_cast<int>(ld_acquire_sys(fl) - epoch) >= 0) break;
        if (it >= kSpinMax || global_ns() - t0 > P.vp_timeout_ns) {
          lost = 1;
          atomicExch(err, 1);
          break;
        }
        __nanosleep(128);
      }
    }
  }
  if (tid == 0) M_S.ib[5] = 0;
  vp::gsync<NT>(bar);
  if (lost) M_S.ib[5] = 1;
  vp::gsync<NT>(bar);
  lost = M_S.ib[5];
  vp::VParams M;
  M.B = P.B; M.V = P.vocab_total; M.Bs = P.vp_maxb;
  M.temperature = P.temperature; M.top_k = P.top_k; M.top_p = P.top_p;
  M.cap = P.cand_cap; M.world = world;
  const long long slot0 = static_cast<long long>(epoch & 1u) * world * P.vp_maxb;
  M.all_cand = reinterpret_cast<const unsigned long long*>(own + P.vp_lcand) + slot0 * P.cand_cap;
  M.all_count = reinterpret_cast<const int*>(own + P.vp_lcount) + slot0;
  M.uniforms = P.uniforms; M.philox_state = P.philox_state;
  M.done_counter = reinterpret_cast<unsigned*>(own + 4);
  M.epoch = reinterpret_cast<unsigned*>(own);
  M.out = P.out; M.row_stats = P.row_stats;
  vp::merge_row<DT, NT>(M, M_S, row, lost != 0, tid, bar);
  vp::gsync<NT>(bar);   // the group's scratch is reused by its next row
}

// The whole vocabulary-parallel step for this rank: stream, local list into
// every rank's exchange buffer, flags, waits, merge and draw.
template <int DT>
__global__ void __launch_bounds__(kT, 1) vp_step_row_kernel(const __grid_constant__ KParams P) {
  row_body<DT, false, 2>(P);
}

}  // namespace rk
}  // namespace ecah
