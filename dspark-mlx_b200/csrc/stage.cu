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
#include <algorithm>

#include "common.cuh"

namespace dsm {
namespace {

constexpr int kStageThreads = 128;

// 8 consecutive elements of a row (k multiple of 8) as floats; zeros past dim
template <typename XT>
__device__ __forceinline__ void load8(const XT* row, int k, int dim, bool vec_ok, float (&v)[8]) {
  if (vec_ok && k + 8 <= dim) {
    if constexpr (sizeof(XT) == 2) {
      const uint4 u = *reinterpret_cast<const uint4*>(row + k);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
    } else {
      const float4 a = *reinterpret_cast<const float4*>(row + k);
      const float4 b = *reinterpret_cast<const float4*>(row + k + 4);
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (k + i < dim) ? load_as_float(row, k + i) : 0.f;
  }
}

struct StageJob {
  const int32_t* perm;  // NULL: row r is token r
  int topk;
  __half* staged;
  int64_t rows_cap;
  float* row_scale;
  const int32_t* n_valid;  // the count of rows to stage (stage_rows_count_kernel only)
};

// One staged row: 16-byte loads, block max, one 16-byte store per 8 columns (the whole CTA).
template <typename XT>
__device__ __forceinline__ void stage_one_row(const XT* __restrict__ x, int64_t n_tokens, int dim, int64_t r,
                                              const StageJob& j, int k_chunks, float* red) {
  const int32_t* __restrict__ perm = j.perm;
  const int topk = j.topk;
  __half* __restrict__ staged = j.staged;
  const int64_t rows_cap = j.rows_cap;
  float* __restrict__ row_scale = j.row_scale;
  int64_t t = perm ? int64_t(perm[r]) / topk : r;
  if (t < 0 || t >= n_tokens) {
    if (threadIdx.x == 0) raise_device_error(DSM_DEV_ERR_TOKEN_RANGE);
    t = 0;
  }
  const XT* row = x + t * dim;
  const bool vec_ok = (dim % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  const int kpad = k_chunks * kChunkK;
  float amax = 0.f;
  for (int k = threadIdx.x * 8; k < dim; k += kStageThreads * 8) {
    float v[8];
    load8(row, k, dim, vec_ok, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __syncthreads();  // red is reused by the next row of a looping CTA
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < kStageThreads / 32; ++i) amax = fmaxf(amax, red[i]);
  int s = 0;
  if (amax > 0.f && isfinite(amax)) {
    int ex;
    frexpf(amax, &ex);  // amax in [2^(ex-1), 2^ex)
    s = 15 - ex;
    s = s < -100 ? -100 : (s > 100 ? 100 : s);
  }
  const float up = ldexpf(1.f, s);
  if (threadIdx.x == 0) row_scale[r] = ldexpf(1.f, -s);
  for (int k = threadIdx.x * 8; k < kpad; k += kStageThreads * 8) {
    float v[8];
    load8(row, k, dim, vec_ok, v);
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 p = __floats2half2_rn(v[2 * i] * up, v[2 * i + 1] * up);
      h[i] = *reinterpret_cast<const uint32_t*>(&p);
    }
    const int c = k / kChunkK, col = k % kChunkK;
    *reinterpret_cast<uint4*>(staged + (int64_t(c) * rows_cap + r) * kStagePitch + col) = make_uint4(h[0], h[1], h[2], h[3]);
  }
}

// One CTA per staged row. Blocks [0, n_rows) serve job a; blocks [n_rows, n_rows + n_rows_b)
// serve job b.
template <typename XT>
__global__ void __launch_bounds__(kStageThreads) stage_rows_kernel(const XT* __restrict__ x, int64_t n_tokens, int dim,
                                                                   int64_t n_rows, StageJob ja, StageJob jb,
                                                                   int k_chunks) {
  __shared__ float red[kStageThreads / 32];
  const bool second = int64_t(blockIdx.x) >= n_rows;
  const int64_t r = second ? int64_t(blockIdx.x) - n_rows : int64_t(blockIdx.x);
  stage_one_row(x, n_tokens, dim, r, second ? jb : ja, k_chunks, red);
}

// Rows r < *j.n_valid (a device count), the CTAs striding over them.
template <typename XT>
__global__ void __launch_bounds__(kStageThreads) stage_rows_count_kernel(const XT* __restrict__ x, int64_t n_tokens,
                                                                         int dim, StageJob j, int k_chunks) {
  __shared__ float red[kStageThreads / 32];
  const int64_t n = *j.n_valid;
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) stage_one_row(x, n_tokens, dim, r, j, k_chunks, red);
}

// One CTA per fp32 row: the row staged as stage_rows_kernel does (row r), then the residual
// x - hi, kept in shared memory, staged with its own power-of-two scale (row n_rows + r).
__global__ void __launch_bounds__(kStageThreads) stage_hilo_kernel(const float* __restrict__ x, int64_t n_rows, int dim,
                                                                   __half* __restrict__ staged, int64_t rows_cap,
                                                                   float* __restrict__ row_scale, int k_chunks) {
  extern __shared__ float res[];  // kpad floats: the residual row
  __shared__ float red[kStageThreads / 32];
  const int64_t r = blockIdx.x;
  const float* row = x + r * dim;
  const int kpad = k_chunks * kChunkK;
  auto row_exp = [&](float amax) {  // power-of-two scale putting amax in [2^14, 2^15)
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int i = 1; i < kStageThreads / 32; ++i) amax = fmaxf(amax, red[i]);
    int s = 0;
    if (amax > 0.f && isfinite(amax)) {
      int ex;
      frexpf(amax, &ex);
      s = 15 - ex;
      s = s < -100 ? -100 : (s > 100 ? 100 : s);
    }
    return s;
  };
  auto store8 = [&](int64_t srow, int k, const float (&v)[8], float up) {
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 p = __floats2half2_rn(v[2 * i] * up, v[2 * i + 1] * up);
      h[i] = *reinterpret_cast<const uint32_t*>(&p);
    }
    const int c = k / kChunkK, col = k % kChunkK;
    *reinterpret_cast<uint4*>(staged + (int64_t(c) * rows_cap + srow) * kStagePitch + col) = make_uint4(h[0], h[1], h[2], h[3]);
  };
  float amax = 0.f;
  for (int k = threadIdx.x; k < dim; k += kStageThreads) amax = fmaxf(amax, fabsf(row[k]));
  const int s1 = row_exp(amax);
  const float up1 = ldexpf(1.f, s1), down1 = ldexpf(1.f, -s1);
  if (threadIdx.x == 0) row_scale[r] = down1;
  float ramax = 0.f;
  for (int k = threadIdx.x * 8; k < kpad; k += kStageThreads * 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (k + i < dim) ? row[k + i] : 0.f;
    store8(r, k, v, up1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float lo = v[i] - __half2float(__float2half_rn(v[i] * up1)) * down1;  // exact difference
      res[k + i] = lo;
      ramax = fmaxf(ramax, fabsf(lo));
    }
  }
  const int s2 = row_exp(ramax);
  const float up2 = ldexpf(1.f, s2);
  if (threadIdx.x == 0) row_scale[n_rows + r] = ldexpf(1.f, -s2);
  __syncthreads();
  for (int k = threadIdx.x * 8; k < kpad; k += kStageThreads * 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = res[k + i];
    store8(n_rows + r, k, v, up2);
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
  DSM_REQUIRE(n_rows < (int64_t(1) << 31), "dsm_stage_rows: too many rows");
  return stage_rows_pair(x, x_dtype, n_tokens, dim, perm, n_rows, topk, staged, rows_cap, row_scale, 0, nullptr, 0,
                         nullptr, stream);
}

extern "C" int dsm_stage_rows_count(const void* x, int x_dtype, int64_t n_tokens, int dim, const int32_t* perm,
                                    int64_t max_rows, int topk, void* staged, int64_t rows_cap, float* row_scale,
                                    const int32_t* n_valid, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(n_valid != nullptr, "dsm_stage_rows_count: n_valid is NULL");
  DSM_REQUIRE(dim > 0 && max_rows >= 0 && n_tokens >= 0, "dsm_stage_rows_count: bad shape");
  DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(max_rows), "dsm_stage_rows_count: rows_cap too small");
  DSM_REQUIRE(x_dtype == DSM_DT_F32 || x_dtype == DSM_DT_BF16, "dsm_stage_rows_count: x must be F32 or BF16");
  DSM_REQUIRE(!perm || topk >= 1, "dsm_stage_rows_count: topk must be >= 1 with a permutation");
  if (max_rows == 0) return DSM_OK;
  DSM_REQUIRE(x && staged && row_scale, "dsm_stage_rows_count: NULL pointer");
  DSM_REQUIRE((reinterpret_cast<uintptr_t>(staged) & 15) == 0, "dsm_stage_rows_count: staged must be 16-byte aligned");
  DSM_REQUIRE(max_rows < (int64_t(1) << 31), "dsm_stage_rows_count: too many rows");
  return stage_rows_pair(x, x_dtype, n_tokens, dim, perm, max_rows, topk, staged, rows_cap, row_scale, 0, nullptr, 0,
                         nullptr, stream, n_valid);
}

extern "C" int dsm_stage_rows_hilo(const float* x, int64_t n_rows, int dim, void* staged, int64_t rows_cap,
                                   float* row_scale, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(!n_rows || (x && staged && row_scale), "dsm_stage_rows_hilo: NULL pointer");
  DSM_REQUIRE((reinterpret_cast<uintptr_t>(staged) & 15) == 0, "dsm_stage_rows_hilo: staged must be 16-byte aligned");
  return stage_rows_hilo(x, n_rows, dim, staged, rows_cap, row_scale, stream);
}

namespace dsm {
int stage_rows_hilo(const float* x, int64_t n_rows, int dim, void* staged, int64_t rows_cap, float* row_scale,
                    void* stream) {
  DSM_REQUIRE(dim > 0 && n_rows >= 0, "stage_rows_hilo: bad shape");
  DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(2 * n_rows), "stage_rows_hilo: rows_cap too small");
  if (n_rows == 0) return DSM_OK;
  const int kc = int(ceil_div(dim, kChunkK));
  const size_t smem = size_t(kc) * kChunkK * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(stage_hilo_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return check_launch("stage_hilo smem attribute");
  stage_hilo_kernel<<<unsigned(n_rows), kStageThreads, smem, as_stream(stream)>>>(
      x, n_rows, dim, static_cast<__half*>(staged), rows_cap, row_scale, kc);
  return check_launch("stage_hilo");
}

int stage_rows_pair(const void* x, int x_dtype, int64_t n_tokens, int dim, const int32_t* perm, int64_t n_rows,
                    int topk, void* staged, int64_t rows_cap, float* row_scale, int64_t n_rows_b, void* staged_b,
                    int64_t rows_cap_b, float* row_scale_b, void* stream, const int32_t* n_valid) {
  const int kc = int(ceil_div(dim, kChunkK));
  const StageJob ja{perm, topk, static_cast<__half*>(staged), rows_cap, row_scale, n_valid};
  const StageJob jb{nullptr, 1, static_cast<__half*>(staged_b), rows_cap_b, row_scale_b, nullptr};
  if (n_valid) {  // job a only, over a device count of at most n_rows rows
    const unsigned grid = unsigned(std::min<int64_t>(n_rows, 8 * int64_t(num_sms())));
    cudaStream_t s = as_stream(stream);
    if (grid == 0) return DSM_OK;
    if (x_dtype == DSM_DT_BF16)
      stage_rows_count_kernel<__nv_bfloat16><<<grid, kStageThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                                            n_tokens, dim, ja, kc);
    else
      stage_rows_count_kernel<float><<<grid, kStageThreads, 0, s>>>(static_cast<const float*>(x), n_tokens, dim, ja,
                                                                    kc);
    return check_launch("stage_rows_count");
  }
  const unsigned blocks = unsigned(n_rows + n_rows_b);
  if (blocks == 0) return DSM_OK;
  cudaStream_t s = as_stream(stream);
  if (x_dtype == DSM_DT_BF16)
    stage_rows_kernel<__nv_bfloat16><<<blocks, kStageThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n_tokens,
                                                                      dim, n_rows, ja, jb, kc);
  else
    stage_rows_kernel<float><<<blocks, kStageThreads, 0, s>>>(static_cast<const float*>(x), n_tokens, dim, n_rows, ja,
                                                              jb, kc);
  return check_launch("stage_rows");
}
}  // namespace dsm
