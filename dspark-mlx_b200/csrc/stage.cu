// Activation staging: the lhs of the grouped expert products.
//
// The reference broadcasts x[N,1,1,dim] against the per-(token, slot) expert ids inside
// gather_mm (dspark_mlx/model/moe.py:158). Here the rows are materialised once, in expert
// order (row r is token perm[r] / topk), in the layout the expert kernels stream with one
// bulk copy per pipeline stage: K-chunk-major, [chunk][row][kStagePitch] halves, chunk c
// holding columns [128c, 128c+128).
//
// Each row is scaled by a power of two 2^s chosen so that its largest magnitude lies in
// [2^14, 2^15): bf16 values then convert to f16 exactly (f16 has 3 more mantissa bits and
// the scaled range sits inside f16's normal range; only entries below 2^-28 of the row
// maximum lose bits), so the f16 tensor-core products see the reference's bf16 operand.
// row_scale[r] = 2^-s undoes it in the epilogue.
#include "common.cuh"

namespace dsm {
namespace {

template <typename XT>
__global__ void __launch_bounds__(256) stage_rows_kernel(const XT* __restrict__ x, int64_t n_tokens, int dim,
                                                         const int32_t* __restrict__ perm, int64_t n_rows, int topk,
                                                         __half* __restrict__ staged, int64_t rows_cap,
                                                         float* __restrict__ row_scale, int k_chunks) {
  const int lane = threadIdx.x & 31;
  const int64_t r = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= n_rows) return;
  int64_t t = perm ? int64_t(perm[r]) / topk : r;
  if (t < 0 || t >= n_tokens) {
    if (lane == 0) raise_device_error(DSM_DEV_ERR_TOKEN_RANGE);
    t = 0;
  }
  const XT* row = x + t * dim;
  float amax = 0.f;
  for (int k = lane; k < dim; k += 32) amax = fmaxf(amax, fabsf(load_as_float(row, k)));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  int s = 0;
  if (amax > 0.f && isfinite(amax)) {
    int ex;
    frexpf(amax, &ex);  // amax in [2^(ex-1), 2^ex)
    s = 15 - ex;
    s = s < -100 ? -100 : (s > 100 ? 100 : s);
  }
  const float up = ldexpf(1.f, s);
  if (lane == 0) row_scale[r] = ldexpf(1.f, -s);
  const int kpad = k_chunks * kChunkK;
  for (int k = lane * 2; k < kpad; k += 64) {
    float v0 = 0.f, v1 = 0.f;
    if (k < dim) v0 = load_as_float(row, k) * up;
    if (k + 1 < dim) v1 = load_as_float(row, k + 1) * up;
    const int c = k / kChunkK, col = k % kChunkK;
    __half2* dst = reinterpret_cast<__half2*>(staged + (int64_t(c) * rows_cap + r) * kStagePitch + col);
    *dst = __floats2half2_rn(v0, v1);
  }
}

}  // namespace
}  // namespace dsm

extern "C" int64_t dsm_stage_rows_cap(int64_t n_rows) { return dsm::ceil_div(n_rows, 8) * 8 + 64; }

extern "C" size_t dsm_stage_bytes(int64_t rows_cap, int k_dim) {
  return size_t(dsm::ceil_div(k_dim, dsm::kChunkK)) * size_t(rows_cap) * dsm::kStagePitch * sizeof(__half);
}

extern "C" int dsm_stage_rows(const void* x, int x_dtype, int64_t n_tokens, int dim, const int32_t* perm,
                              int64_t n_rows, int topk, void* staged, int64_t rows_cap, float* row_scale,
                              void* stream) {
  using namespace dsm;
  DSM_REQUIRE(dim > 0 && n_rows >= 0 && n_tokens >= 0, "dsm_stage_rows: bad shape");
  DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(n_rows), "dsm_stage_rows: rows_cap smaller than dsm_stage_rows_cap(n_rows)");
  DSM_REQUIRE(x_dtype == DSM_DT_F32 || x_dtype == DSM_DT_BF16, "dsm_stage_rows: x must be F32 or BF16");
  DSM_REQUIRE(!perm || topk >= 1, "dsm_stage_rows: topk must be >= 1 with a permutation");
  if (n_rows == 0) return DSM_OK;
  DSM_REQUIRE(x && staged && row_scale, "dsm_stage_rows: NULL pointer");
  DSM_REQUIRE((reinterpret_cast<uintptr_t>(staged) & 15) == 0, "dsm_stage_rows: staged must be 16-byte aligned");
  const int kc = int(ceil_div(dim, kChunkK));
  const unsigned blocks = unsigned(ceil_div(n_rows, 8));
  cudaStream_t s = as_stream(stream);
  if (x_dtype == DSM_DT_BF16)
    stage_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n_tokens, dim, perm,
                                                            n_rows, topk, static_cast<__half*>(staged), rows_cap,
                                                            row_scale, kc);
  else
    stage_rows_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(x), n_tokens, dim, perm, n_rows, topk,
                                                    static_cast<__half*>(staged), rows_cap, row_scale, kc);
  return check_launch("stage_rows");
}
