// Weighted combine: y = sum_k o[t, k] * w[t, k] (fp32) + shared[t] (fp32) -> y dtype
// (dspark_mlx/model/moe.py:159-161). o rows are in expert-sorted order; inv maps the
// (token, slot) pair to its sorted row. Slots are summed in ascending slot order.
#include "common.cuh"

namespace dsm {
namespace {

template <typename YT>
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ o, const int32_t* __restrict__ inv,
                                                      const float* __restrict__ w, int64_t n_tokens, int topk,
                                                      int dim, const float* __restrict__ shared, YT* __restrict__ y) {
  // grid (tokens, column blocks): one thread per 4 consecutive columns of one token
  const int64_t t = blockIdx.x;
  const int32_t* it = inv + t * topk;
  const float* wt = w + t * topk;
  for (int d = (blockIdx.y * blockDim.x + threadIdx.x) * 4; d < dim; d += gridDim.y * blockDim.x * 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < topk; ++s) {
      const float ws = wt[s];
      const float* row = o + int64_t(it[s]) * dim + d;
      if (d + 3 < dim && (dim & 3) == 0) {
        const float4 v = *reinterpret_cast<const float4*>(row);
        acc[0] += v.x * ws;
        acc[1] += v.y * ws;
        acc[2] += v.z * ws;
        acc[3] += v.w * ws;
      } else {
        for (int c = 0; c < 4 && d + c < dim; ++c) acc[c] += row[c] * ws;
      }
    }
    for (int c = 0; c < 4 && d + c < dim; ++c) {
      float v = acc[c];
      if (shared) v += shared[t * dim + d + c];
      if constexpr (sizeof(YT) == 2)
        y[t * dim + d + c] = __float2bfloat16_rn(v);
      else
        y[t * dim + d + c] = v;
    }
  }
}

}  // namespace
}  // namespace dsm

extern "C" int dsm_combine(const float* o_sorted, const int32_t* inv, const float* route_weights, int64_t n_tokens,
                           int topk, int dim, const float* shared_rows, void* y, int y_dtype, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(n_tokens >= 0 && topk >= 1 && dim > 0, "dsm_combine: bad shape");
  DSM_REQUIRE(y_dtype == DSM_DT_F32 || y_dtype == DSM_DT_BF16, "dsm_combine: y must be F32 or BF16");
  if (n_tokens == 0) return DSM_OK;
  DSM_REQUIRE(o_sorted && inv && route_weights && y, "dsm_combine: NULL pointer");
  DSM_REQUIRE(n_tokens < (int64_t(1) << 31), "dsm_combine: too many tokens");
  cudaStream_t s = as_stream(stream);
  const int threads = 128;
  const dim3 grid(unsigned(n_tokens), unsigned(ceil_div(ceil_div(dim, 4), threads)));
  if (y_dtype == DSM_DT_BF16)
    combine_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(o_sorted, inv, route_weights, n_tokens, topk,
                                                                         dim, shared_rows,
                                                                         static_cast<__nv_bfloat16*>(y));
  else
    combine_kernel<float><<<grid, threads, 0, s>>>(o_sorted, inv, route_weights, n_tokens, topk, dim,
                                                                 shared_rows, static_cast<float*>(y));
  return check_launch("combine");
}
