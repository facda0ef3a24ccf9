// Diagnostic entry point of libecah_sampler.so: the quotient the kernels use
// for softmax masses (quot_rn: reciprocal plus one correction step) against
// the IEEE quotient __fdiv_rn, over every input of a dtype and a list of
// temperatures.  The reference divides with torch (`logits / temperature`,
// ecahlang/main.py:170), an IEEE float32 divide; the kernels' masses are
// exact only where the two agree.

#include "common.cuh"

namespace ecah {

// Per temperature t, over finite inputs whose IEEE quotient is a normal
// float32 (|q| >= 2^-126): counts[3 t] = quotients more than one unit in the
// last place away from it, counts[3 t + 1] = quotients exactly one unit away;
// counts[3 t + 2] = the other differences (the sign of a zero, subnormal
// quotients, non-finite inputs), which the masses never see: a subnormal z
// lies 87 or more below any row max of a sampled row.
template <int DT>
__global__ void quotient_check_kernel(const float* T, int nT, unsigned long long* counts) {
  const unsigned long long n = (DT == ECAH_DTYPE_F32) ? (1ull << 32) : (1ull << 16);
  const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
  for (int t = 0; t < nT; ++t) {
    const float Tv = T[t];
    const float rT = __frcp_rn(Tv);
    unsigned long long bad = 0, ulp1 = 0, other = 0;
    for (unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride) {
      const float y = DType<DT>::to_f32(static_cast<uint32_t>(i));
      const float a = quot_rn(y, Tv, rT);
      const float b = __fdiv_rn(y, Tv);
      if (__float_as_uint(a) == __float_as_uint(b)) continue;
      if (a != a && b != b) continue;   // both NaN
      const bool normal = isfinite(y) && fabsf(b) >= 1.17549435e-38f && isfinite(b);
      if (normal && a != b) {
        const int d = static_cast<int>(__float_as_uint(a)) - static_cast<int>(__float_as_uint(b));
        if (d == 1 || d == -1) ++ulp1;
        else ++bad;
      } else {
        ++other;
      }
    }
    bad = __reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(bad));
    ulp1 = __reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(ulp1));
    other = __reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(other));
    if ((threadIdx.x & 31) == 0) {
      if (bad) atomicAdd(&counts[3 * t], bad);
      if (ulp1) atomicAdd(&counts[3 * t + 1], ulp1);
      if (other) atomicAdd(&counts[3 * t + 2], other);
    }
  }
}

}  // namespace ecah

using namespace ecah;

extern "C" int ecah_quotient_mismatches(int32_t dtype, const float* temperature, int32_t n_temperature,
                                        unsigned long long* counts, void* stream) {
  if (n_temperature < 0) return ECAH_ERR_SHAPE;
  if (n_temperature == 0) return ECAH_OK;
  if (!temperature || !counts) return ECAH_ERR_NULL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(counts, 0, sizeof(unsigned long long) * 3 * n_temperature, s) != cudaSuccess)
    return ECAH_ERR_LAUNCH;
  switch (dtype) {
    case ECAH_DTYPE_F16: quotient_check_kernel<ECAH_DTYPE_F16><<<64, 1024, 0, s>>>(temperature, n_temperature, counts); break;
    case ECAH_DTYPE_BF16: quotient_check_kernel<ECAH_DTYPE_BF16><<<64, 1024, 0, s>>>(temperature, n_temperature, counts); break;
    case ECAH_DTYPE_F32: quotient_check_kernel<ECAH_DTYPE_F32><<<1184, 1024, 0, s>>>(temperature, n_temperature, counts); break;
    default: return ECAH_ERR_DTYPE;
  }
  return cudaGetLastError() == cudaSuccess ? ECAH_OK : ECAH_ERR_LAUNCH;
}
