// The Qwen3 draft layer's glue around its attention and MLP (dspark_mlx/arch/qwen3.py:157-176):
//
//   dsm_add_rms_norm  s = x + delta, rounded to the activation dtype as MLX adds two arrays
//                     (the residual add; delta optional), and y = RMSNorm(s) * weight
//                     (norm_rope.py:22-39: fp32 normalisation, fp32 weight, cast back).
//                     s and y are each optional. One CTA per row, the row held in shared
//                     memory between the sum of squares and the scaling.
#include "common.cuh"

namespace dsm {
namespace {

constexpr int kNormThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rms_norm_kernel(const T* __restrict__ x,
                                                                    const T* __restrict__ delta, int dim,
                                                                    const float* __restrict__ weight, float eps,
                                                                    T* __restrict__ sum_out, T* __restrict__ norm_out) {
  extern __shared__ float row[];
  __shared__ float red[kNormThreads / 32];
  const int64_t off = int64_t(blockIdx.x) * dim;
  float sq = 0.f;
  for (int c = threadIdx.x; c < dim; c += kNormThreads) {
    float v = ld_f(x, off + c);
    if (delta) v = rnd<T>(v + ld_f(delta, off + c));
    if (sum_out) sum_out[off + c] = st_f<T>(v);
    row[c] = v;
    sq = fmaf(v, v, sq);
  }
  if (!norm_out) return;  // uniform across the CTA: no barrier is skipped by part of it
#pragma unroll
  for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
  const float rs = rsqrtf(tot / float(dim) + eps);
  for (int c = threadIdx.x; c < dim; c += kNormThreads)
    norm_out[off + c] = st_f<T>(__fmul_rn(weight[c], __fmul_rn(row[c], rs)));
}

}  // namespace
}  // namespace dsm

using namespace dsm;

extern "C" int dsm_add_rms_norm(const void* x, const void* delta, int dtype, int64_t n_rows, int dim,
                                const float* weight, float eps, void* sum_out, void* norm_out, void* stream) {
  DSM_REQUIRE(n_rows >= 0 && dim > 0 && dim <= 48 * 1024, "dsm_add_rms_norm: bad shape");
  DSM_REQUIRE(dtype == DSM_DT_F32 || dtype == DSM_DT_BF16, "dsm_add_rms_norm: dtype must be F32 or BF16");
  DSM_REQUIRE(n_rows <= 0x7fffffff, "dsm_add_rms_norm: too many rows");
  if (n_rows == 0) return DSM_OK;
  DSM_REQUIRE(x && (sum_out || norm_out) && (!norm_out || weight), "dsm_add_rms_norm: NULL pointer");
  const size_t smem = size_t(dim) * 4;
  cudaStream_t s = as_stream(stream);
  if (dtype == DSM_DT_BF16) {
    auto k = add_rms_norm_kernel<__nv_bfloat16>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
      return check_launch("add_rms_norm smem attribute");
    using B = __nv_bfloat16;
    k<<<unsigned(n_rows), kNormThreads, smem, s>>>(static_cast<const B*>(x), static_cast<const B*>(delta), dim, weight,
                                                   eps, static_cast<B*>(sum_out), static_cast<B*>(norm_out));
  } else {
    auto k = add_rms_norm_kernel<float>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
      return check_launch("add_rms_norm smem attribute");
    k<<<unsigned(n_rows), kNormThreads, smem, s>>>(static_cast<const float*>(x), static_cast<const float*>(delta), dim,
                                                   weight, eps, static_cast<float*>(sum_out),
                                                   static_cast<float*>(norm_out));
  }
  return check_launch("add_rms_norm");
}
