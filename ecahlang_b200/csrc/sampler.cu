// Host launcher and small kernels of libecah_sampler.so (C ABI in
// include/ecah_sampler.h).  The sampler kernels are the row kernel
// (row_kernel.cuh: fp16/bf16 logits without additive penalties, given the
// full workspace) and the cluster kernel (sampler_kernel.cuh: everything
// else); stream_kernel.cuh writes probs_out after the row kernel.

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "row_kernel.cuh"
#include "vp_kernel.cuh"
#include "vp_dist.cuh"

namespace ecah {

// ------------------------------------------------------ vocab-parallel reset
// Exchange-buffer header words: [0] step epoch, [1] rows finished in the
// step, [2] error (a wait ran out).
__global__ void vp_reset_kernel(unsigned* hdr, unsigned epoch) {
  if (threadIdx.x == 0) {
    hdr[0] = epoch;
    hdr[1] = 0u;
    hdr[2] = 0u;
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
  int fx_log2;
};

static constexpr size_t kMaxDynSmem = 128 * 1024;
// the cluster kernel's workspace: the Philox completion counter
static constexpr size_t kMinWorkspace = 256;

// SM count of the current device, looked up once per device.
static int device_sms() {
  constexpr int kMaxDev = 64;
  static int cache[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 0;
  if (cache[dev] > 0) return cache[dev];
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  cache[dev] = sms;
  return sms;
}

// Workspace header: [0, 256) the Philox completion counter and the error
// word; [256, 4096) one arrival counter per row split over several CTAs.
// Both are left at zero by every launch, at fixed offsets for any batch.
static constexpr size_t kHeaderBytes = 4096;
static constexpr int kMinParts = 4;
static constexpr int kMaxSplitRows = static_cast<int>((kHeaderBytes - kMinWorkspace) / sizeof(unsigned));

// CTAs per row of the row kernel: enough to occupy the SMs of the current
// device when the batch is small, at most one per 16384-entry round.
static int row_parts(long long B, int V) {
  const int R = (V + rk::kRound - 1) / rk::kRound;
  const int sms = device_sms();
  if (B <= 0 || B > kMaxSplitRows || sms <= 0 || V > rk::kMaxRounds * rk::kRound) return 1;
  // two or three parts per row cost more in the exchange than they save
  const long long p = sms / B;
  return static_cast<int>(p < kMinParts ? 1 : (p > R ? R : p));
}

static size_t a256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// bytes of the per-part regions of a row kernel launch at batch B (0 when
// its rows are not split)
static size_t parts_bytes(long long B, int V) {
  const size_t pp = static_cast<size_t>(row_parts(B, V));
  if (pp < 2) return 0;
  const size_t b = static_cast<size_t>(B);
  return a256(b * pp * sizeof(rk::PartHdr)) + a256(b * pp * rk::kCB * sizeof(unsigned long long)) +
         a256(b * rk::kMaxRounds * rk::kNW * sizeof(float2));
}

// Row-kernel workspace regions after the header, each 256-byte aligned: the
// finished-row data of the probability kernel, then, for rows split over
// several CTAs, the parts' headers, candidates and segment masses.  Every
// region is written before it is read within a launch.
struct RowLayout {
  int NC, parts;                    // 8192-entry chunks per row (probability kernel)
  size_t fin, base_total;           // base_total: without the split-row regions
  size_t hdr, pcand, pseg, total;
};

static bool row_layout(long long B, int V, RowLayout* L) {
  if (B < 0 || V < 1 || V > rk::kMaxRounds * rk::kRound) return false;
  const size_t b = static_cast<size_t>(B);
  size_t off = kHeaderBytes;
  L->fin = off; off += a256(b * sizeof(RowFin));
  L->NC = (V + kSCH - 1) / kSCH;
  L->base_total = off;
  L->parts = row_parts(B, V);
  const size_t pp = static_cast<size_t>(L->parts);
  L->hdr = L->pcand = L->pseg = 0;
  if (pp > 1) {
    L->hdr = off; off += a256(b * pp * sizeof(rk::PartHdr));
    L->pcand = off; off += a256(b * pp * rk::kCB * sizeof(unsigned long long));
    L->pseg = off; off += a256(b * rk::kMaxRounds * rk::kNW * sizeof(float2));
  }
  L->total = off;
  return true;
}

static bool k16_dtype(int dtype) { return dtype == ECAH_DTYPE_F16 || dtype == ECAH_DTYPE_BF16; }

static bool make_plan(int dtype, int V, unsigned flags, Plan* p) {
  const int kb = (dtype == ECAH_DTYPE_F32) ? 32 : 16;   // additive penalties stay in the model dtype
  const int ksz = kb / 8;
  const int kpv = 16 / ksz;                       // keys per 16-byte vector
  const int target = (kb == 16) ? 20480 : 10240;  // keys per CTA aimed for (~40 KB)
  int CL = (V + target - 1) / target;
  if (CL < 1) CL = 1;
  if (CL > 8) CL = 16;
  int CH = (V + CL - 1) / CL;
  CH = (CH + 7) / 8 * 8;
  const size_t smem = static_cast<size_t>(CH) * ksz;
  if (smem > kMaxDynSmem) return false;
  if ((CH + 32 * kpv - 1) / (32 * kpv) > kMaxSeg) return false;
  // fixed-point level-0 masses: a [bin][lane] slot sums at most ceil(CH/32)
  // masses <= 1, so scale * ceil(CH/32) must stay below 2^32 (and <= 2^22)
  const long long per_lane = (CH + 31) / 32;
  int fx = 22;
  while (fx > 0 && (per_lane << fx) >= (1ll << 32)) --fx;
  p->CL = CL; p->CH = CH; p->kb = kb; p->smem = smem; p->fx_log2 = fx;
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

// cudaFuncSetAttribute once per (kernel, device, value): the attribute is a
// property of the kernel on a device, so later launches skip the call.
// forget_smem drops the remembered values (a launch that failed sets them
// again: after cudaDeviceReset the kernels come back without them).
static std::mutex g_smem_mu;
static constexpr int kSmemSlots = 64;
static KernelFn g_smem_fn[kSmemSlots];
static int g_smem_dev[kSmemSlots], g_smem_val[kSmemSlots];
static int g_smem_used = 0;

static void forget_smem() {
  std::lock_guard<std::mutex> lock(g_smem_mu);
  g_smem_used = 0;
}

static cudaError_t set_smem_once(KernelFn fn, int smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_smem_mu);
  KernelFn* fns = g_smem_fn;
  int* devs = g_smem_dev;
  int* vals = g_smem_val;
  int& used = g_smem_used;
  constexpr int kSlots = kSmemSlots;
  for (int i = 0; i < used; ++i)
    if (fns[i] == fn && devs[i] == dev && vals[i] >= smem) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  for (int i = 0; i < used; ++i)
    if (fns[i] == fn && devs[i] == dev) { vals[i] = smem; return cudaSuccess; }
  if (used < kSlots) { fns[used] = fn; devs[used] = dev; vals[used] = smem; ++used; }
  return cudaSuccess;
}

size_t ecah_sampler_workspace_bytes(int32_t batch, int32_t vocab, int32_t dtype) {
  RowLayout L;
  if (!k16_dtype(dtype) || !row_layout(batch, vocab, &L)) return kMinWorkspace;
  // any launch of at most `batch` rows fits: the finished-row region grows
  // with the batch, the split-row regions peak at some smaller batch
  size_t split = 0;
  const int top = batch < kMaxSplitRows ? batch : kMaxSplitRows;
  for (int b = 1; b <= top; ++b) split = std::max(split, parts_bytes(b, vocab));
  return L.base_total + split;
}

// Not exported: the least workspace any launch accepts (the cluster kernel's).
size_t ecah_internal_min_workspace_bytes(void) { return kMinWorkspace; }

int ecah_sampler_launch(const ecah_sampler_args* a, void* stream) {
  if (!a) return ECAH_ERR_NULL;
  if (a->abi_version != ECAH_SAMPLER_ABI_VERSION) return ECAH_ERR_ABI;
  if (a->dtype < ECAH_DTYPE_F16 || a->dtype > ECAH_DTYPE_F32) return ECAH_ERR_DTYPE;
  if (a->batch < 0 || a->vocab < 1 || a->row_stride < a->vocab) return ECAH_ERR_SHAPE;
  if (a->batch == 0) return ECAH_OK;
  if (!a->logits || !a->temperature || !a->top_k || !a->top_p || !a->out) return ECAH_ERR_NULL;
  if (!a->uniforms && !a->philox_state) return ECAH_ERR_NULL;
  if (a->row_slot && (!a->slot_len || !a->hist_tok || !a->hist_cnt || a->hist_cap < 0)) return ECAH_ERR_NULL;
  if (!a->workspace || a->workspace_bytes < kMinWorkspace) return ECAH_ERR_WORKSPACE;
  if (a->row_index && a->logit_rows < 1) return ECAH_ERR_SHAPE;

  KParams P = {};
  P.logits = a->logits;
  P.row_stride = a->row_stride;
  P.row_index = a->row_index;
  P.logit_rows = a->row_index ? a->logit_rows : a->batch;
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
  const int es = elem_size(a->dtype);
  P.vec_ok = (reinterpret_cast<uintptr_t>(a->logits) % 16 == 0) && ((a->row_stride * es) % 16 == 0);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  // row kernel: 16-bit keys; one CTA per row, or a row split over several
  // CTAs when the batch leaves SMs idle
  RowLayout L;
  const bool k16 = k16_dtype(a->dtype);   // additive penalties keep the logits in the model dtype
  if (k16 && row_layout(a->batch, a->vocab, &L) && a->workspace_bytes >= L.total) {
    unsigned char* ws = static_cast<unsigned char*>(a->workspace);
    P.NC = L.NC;
    P.ws_fin = ws + L.fin;
    P.parts = L.parts;
    P.part_arrive = L.parts > 1 ? reinterpret_cast<unsigned*>(ws + kMinWorkspace) : nullptr;
    P.part_hdr = L.parts > 1 ? ws + L.hdr : nullptr;
    P.part_cand = L.parts > 1 ? reinterpret_cast<unsigned long long*>(ws + L.pcand) : nullptr;
    P.part_seg = L.parts > 1 ? reinterpret_cast<float2*>(ws + L.pseg) : nullptr;
    const int smem = static_cast<int>(sizeof(rk::RSmem));
    const int sms = device_sms();
    if (sms <= 0) return ECAH_ERR_LAUNCH;
    const long long units = static_cast<long long>(a->batch) * L.parts;
    const dim3 grid(static_cast<unsigned>(units < sms ? units : sms));
    const dim3 all(static_cast<unsigned>(static_cast<long long>(a->batch) * L.NC));
    KernelFn fn = nullptr;
    if (a->dtype == ECAH_DTYPE_F16)
      fn = L.parts > 1 ? rk::row_sample_kernel<ECAH_DTYPE_F16, true> : rk::row_sample_kernel<ECAH_DTYPE_F16, false>;
    else
      fn = L.parts > 1 ? rk::row_sample_kernel<ECAH_DTYPE_BF16, true> : rk::row_sample_kernel<ECAH_DTYPE_BF16, false>;
    if (set_smem_once(fn, smem) != cudaSuccess)
      return ECAH_ERR_LAUNCH;
    fn<<<grid, rk::kT, smem, s>>>(P);
    if (cudaPeekAtLastError() != cudaSuccess) {
      cudaGetLastError();
      forget_smem();
      if (set_smem_once(fn, smem) != cudaSuccess) return ECAH_ERR_LAUNCH;
      fn<<<grid, rk::kT, smem, s>>>(P);
    }
    if (a->probs_out) {
      if (a->dtype == ECAH_DTYPE_F16) stream_probs_kernel<ECAH_DTYPE_F16><<<all, kThreads, 0, s>>>(P);
      else stream_probs_kernel<ECAH_DTYPE_BF16><<<all, kThreads, 0, s>>>(P);
    }
    return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
  }

  // cluster kernel
  Plan plan;
  if (!make_plan(a->dtype, a->vocab, a->flags, &plan)) return ECAH_ERR_SHAPE;
  if (static_cast<long long>(a->batch) * plan.CL > 0x7FFFFFFFLL) return ECAH_ERR_SHAPE;
  P.CL = plan.CL;
  P.CH = plan.CH;
  P.fx_scale = ldexpf(1.0f, plan.fx_log2);
  P.fx_inv = ldexpf(1.0f, -plan.fx_log2);

  KernelFn fn = pick_kernel(a->dtype, plan.kb);
  cudaError_t e = set_smem_once(fn, static_cast<int>(plan.smem));
  if (e != cudaSuccess) return ECAH_ERR_LAUNCH;
  if (plan.CL > 8) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return ECAH_ERR_LAUNCH;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a->batch * plan.CL), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
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

// the checks both vocab-parallel entry points share
static int vp_check(const ecah_vp_args* a) {
  if (!a) return ECAH_ERR_NULL;
  if (a->abi_version != ECAH_SAMPLER_ABI_VERSION) return ECAH_ERR_ABI;
  if (!k16_dtype(a->dtype)) return ECAH_ERR_DTYPE;
  if (a->batch < 0 || a->vocab < 1 || a->vocab_local < 1 || a->vocab_local > rk::kMaxRounds * rk::kRound ||
      a->vocab_offset < 0 ||
      static_cast<long long>(a->vocab_offset) + a->vocab_local > a->vocab || a->row_stride < a->vocab_local ||
      a->cand_cap < 1 || a->world < 1 || a->world > 64 || static_cast<long long>(a->world) * a->cand_cap > vp::kMaxMerged)
    return ECAH_ERR_SHAPE;
  if (a->batch > 0 && (!a->temperature || !a->top_k || !a->top_p)) return ECAH_ERR_NULL;
  return ECAH_OK;
}

// the row kernel's stream and candidates over a slice (P.V = its length)
static KParams vp_kparams(const ecah_vp_args* a) {
  KParams P = {};
  P.logits = a->logits;
  P.row_stride = a->row_stride;
  P.B = a->batch;
  P.V = a->vocab_local;
  P.temperature = a->temperature;
  P.top_k = a->top_k;
  P.top_p = a->top_p;
  P.rep_factor = a->rep_factor;
  P.row_slot = a->row_slot;
  P.slot_len = a->slot_len;
  P.hist_tok = a->hist_tok;
  P.hist_cnt = a->hist_cnt;
  P.hist_mval = a->hist_mval;
  P.hist_cap = a->hist_cap;
  P.num_slots = a->num_slots;
  P.vec_ok = (reinterpret_cast<uintptr_t>(a->logits) % 16 == 0) && ((a->row_stride * 2) % 16 == 0);
  P.vocab_offset = a->vocab_offset;
  P.vocab_total = a->vocab;
  P.cand_cap = a->cand_cap;
  return P;
}

int ecah_vp_local(const ecah_vp_args* a, void* stream) {
  const int st = vp_check(a);
  if (st != ECAH_OK) return st;
  if (a->batch == 0) return ECAH_OK;
  if (!a->logits || !a->cand || !a->cand_count) return ECAH_ERR_NULL;
  if (a->row_slot && (!a->slot_len || !a->hist_tok || !a->hist_cnt || a->hist_cap < 0)) return ECAH_ERR_NULL;
  KParams P = vp_kparams(a);
  P.vp_cand = reinterpret_cast<unsigned long long*>(a->cand);
  P.vp_count = a->cand_count;
  const int smem = static_cast<int>(sizeof(rk::RSmem));
  const int sms = device_sms();
  if (sms <= 0) return ECAH_ERR_LAUNCH;
  const dim3 grid(static_cast<unsigned>(a->batch < sms ? a->batch : sms));
  KernelFn fn = a->dtype == ECAH_DTYPE_F16 ? rk::vp_local_row_kernel<ECAH_DTYPE_F16> : rk::vp_local_row_kernel<ECAH_DTYPE_BF16>;
  if (set_smem_once(fn, smem) != cudaSuccess) return ECAH_ERR_LAUNCH;
  fn<<<grid, rk::kT, smem, reinterpret_cast<cudaStream_t>(stream)>>>(P);
  return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

// Exchange-buffer layout of the fused step (the same on every rank).
struct VpXLayout {
  long long flag, count, cand, total;
};
static VpXLayout vp_xlayout(long long maxb, long long world, long long cap) {
  auto al = [](long long x) { return (x + 255) & ~255LL; };
  VpXLayout L;
  long long off = 256;   // header: epoch, finished-row counter, error word
  L.flag = off; off += al(4 * world * maxb);
  L.count = off; off += al(4 * 2 * world * maxb);
  L.cand = off; off += al(8 * 2 * world * maxb * cap);
  L.total = off;
  return L;
}

size_t ecah_vp_exchange_bytes(int32_t max_batch, int32_t world, int32_t cand_cap) {
  if (max_batch < 1 || world < 1 || world > 64 || cand_cap < 1) return 0;
  return static_cast<size_t>(vp_xlayout(max_batch, world, cand_cap).total);
}

int ecah_vp_step(const ecah_vp_args* a, const ecah_vp_peers* x, void* stream) {
  const int st = vp_check(a);
  if (st != ECAH_OK) return st;
  if (!x) return ECAH_ERR_NULL;
  if (x->rank < 0 || x->rank >= a->world || x->max_batch < a->batch) return ECAH_ERR_SHAPE;
  if (a->batch == 0) return ECAH_OK;
  if (!a->logits || !a->out || !x->base) return ECAH_ERR_NULL;
  if (!a->uniforms && !a->philox_state) return ECAH_ERR_NULL;
  if (a->row_slot && (!a->slot_len || !a->hist_tok || !a->hist_cnt || a->hist_cap < 0)) return ECAH_ERR_NULL;
  KParams P = vp_kparams(a);
  const VpXLayout L = vp_xlayout(x->max_batch, a->world, a->cand_cap);
  P.vp_base = x->base;
  P.vp_world = a->world;
  P.vp_rank = x->rank;
  P.vp_maxb = x->max_batch;
  P.vp_lflag = L.flag;
  P.vp_lcount = L.count;
  P.vp_lcand = L.cand;
  P.vp_timeout_ns = static_cast<unsigned long long>(x->timeout_us) * 1000ull;
  P.uniforms = a->uniforms;
  P.philox_state = reinterpret_cast<unsigned long long*>(a->philox_state);
  P.out = a->out;
  P.row_stats = a->row_stats;
  const int smem = static_cast<int>(sizeof(rk::RSmem));
  const int sms = device_sms();
  if (sms <= 0) return ECAH_ERR_LAUNCH;
  const dim3 grid(static_cast<unsigned>(a->batch < sms ? a->batch : sms));
  KernelFn fn = a->dtype == ECAH_DTYPE_F16 ? rk::vp_step_row_kernel<ECAH_DTYPE_F16> : rk::vp_step_row_kernel<ECAH_DTYPE_BF16>;
  if (set_smem_once(fn, smem) != cudaSuccess) return ECAH_ERR_LAUNCH;
  fn<<<grid, rk::kT, smem, reinterpret_cast<cudaStream_t>(stream)>>>(P);
  return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

int ecah_vp_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return ECAH_ERR_NULL;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return ECAH_ERR_LAUNCH;
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return ECAH_ERR_LAUNCH;
  }
  return ECAH_OK;
}

int ecah_vp_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return ECAH_ERR_NULL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

int ecah_vp_ipc_close(void* ptr) {
  if (!ptr) return ECAH_ERR_NULL;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

int ecah_vp_ipc_free(void* ptr) {
  if (!ptr) return ECAH_ERR_NULL;
  return cudaFree(ptr) == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

int ecah_vp_reset(void* own_buffer, uint32_t epoch, void* stream) {
  if (!own_buffer) return ECAH_ERR_NULL;
  vp_reset_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(static_cast<unsigned*>(own_buffer), epoch);
  return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

int ecah_vp_dist_pass(const ecah_vp_args* a, int32_t rank, int32_t pass, const int32_t* rows, int32_t nrows,
                      const void* in, void* out, void* stream) {
  const int st = vp_check(a);
  if (st != ECAH_OK) return st;
  const bool combine = pass >= 11 && pass <= 15;
  if (!((pass >= 1 && pass <= 5) || combine) || nrows < 0 || rank < 0 || rank >= a->world) return ECAH_ERR_SHAPE;
  if (nrows == 0) return ECAH_OK;
  if (!rows || !out || (pass != 1 && !in)) return ECAH_ERR_NULL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (combine) {
    if (pass == 15 && !a->out) return ECAH_ERR_NULL;
    if (pass == 14 && !a->uniforms && !a->philox_state) return ECAH_ERR_NULL;
    vd::CParams C = {};
    C.temperature = a->temperature;
    C.top_k = a->top_k;
    C.top_p = a->top_p;
    C.uniforms = a->uniforms;
    C.philox_state = a->philox_state;
    C.out = a->out;
    C.B = a->batch;
    C.vocab = a->vocab;
    C.world = a->world;
    C.rank = rank;
    C.pass = pass - 10;
    C.rows = rows;
    C.n = nrows;
    C.G = static_cast<const float*>(in);
    C.S = static_cast<float*>(out);
    vd::vp_dist_combine_kernel<<<nrows, 32, 0, s>>>(C);
    return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
  }
  if (!a->logits) return ECAH_ERR_NULL;
  if (a->row_slot && (!a->slot_len || !a->hist_tok || !a->hist_cnt || a->hist_cap < 0)) return ECAH_ERR_NULL;
  vd::DParams D = {};
  D.P = vp_kparams(a);
  D.pass = pass;
  D.rows = rows;
  D.n = nrows;
  D.gin = static_cast<const float*>(in);
  D.gout = static_cast<float*>(out);
  if (a->dtype == ECAH_DTYPE_F16) vd::vp_dist_kernel<ECAH_DTYPE_F16><<<nrows, vd::kDT, 0, s>>>(D);
  else vd::vp_dist_kernel<ECAH_DTYPE_BF16><<<nrows, vd::kDT, 0, s>>>(D);
  return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}

int ecah_vp_merge(const ecah_vp_args* a, void* stream) {
  const int st = vp_check(a);
  if (st != ECAH_OK) return st;
  if (a->batch == 0) return ECAH_OK;
  if (!a->all_cand || !a->all_count || !a->out) return ECAH_ERR_NULL;
  if (!a->uniforms && !a->philox_state) return ECAH_ERR_NULL;
  if (!a->workspace || a->workspace_bytes < kMinWorkspace) return ECAH_ERR_WORKSPACE;
  vp::VParams P = {};
  P.B = a->batch; P.V = a->vocab; P.Bs = a->batch;
  P.temperature = a->temperature; P.top_k = a->top_k; P.top_p = a->top_p;
  P.cap = a->cand_cap; P.world = a->world;
  P.all_cand = reinterpret_cast<const unsigned long long*>(a->all_cand);
  P.all_count = a->all_count;
  P.uniforms = a->uniforms;
  P.philox_state = reinterpret_cast<unsigned long long*>(a->philox_state);
  P.done_counter = reinterpret_cast<unsigned*>(a->workspace);
  P.out = a->out;
  P.row_stats = a->row_stats;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (a->dtype == ECAH_DTYPE_F16) vp::vp_merge_kernel<ECAH_DTYPE_F16><<<a->batch, vp::kMT, 0, s>>>(P);
  else vp::vp_merge_kernel<ECAH_DTYPE_BF16><<<a->batch, vp::kMT, 0, s>>>(P);
  return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
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
