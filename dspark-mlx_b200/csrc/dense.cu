// A dense SwiGLU MLP as one call: the Qwen3 draft layer's MLP (dspark_mlx/arch/qwen3.py:146-154,
// down(silu(gate(x)) * up(x))) and, in general, one expert applied to every row
// (dspark_mlx/model/moe.py:82-97). Stage x, gate/up with the activation fused, down, cast.
//
// A dense layer with few tokens has few weight row tiles for its down product (hidden / 128
// of them), each with a long K (inter). Run whole, they leave most SMs idle. For the
// tensor-memory formats the down product is split along K: every (row tile, K range) unit
// converts its weight tiles once, for up to 128 token rows, and writes an fp32 partial slab.
// reduce_splits_kernel then adds the slabs in split order, which is fixed, so the result
// does not depend on scheduling. It applies the bf16 rounding of the reference's products
// and casts to the output dtype.
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace dsm {

float h_scale_for(int act, float limit) {
  // |h| <= limit^2 under the clamp; keep f16 headroom otherwise
  if (act == DSM_ACT_SWIGLU_CLAMP && limit > 0.f && limit * limit < 30000.f) return 1.f;
  return 1.f / 256.f;
}

namespace {

constexpr int kMaxSplits = 8;
constexpr int64_t kSplitCtaBound = 160;  // at least the SM count of the part: sizes the workspace

template <typename YT>
__global__ void __launch_bounds__(256) reduce_splits_kernel(const float* __restrict__ parts, int n_splits,
                                                            int64_t stride, int64_t count, int round,
                                                            YT* __restrict__ y) {
  // four consecutive elements per thread; count and stride are multiples of 4 (dim % 4 == 0).
  // Every slab's load is issued before the first add (one memory latency, not n_splits), and
  // the adds keep split order.
  for (int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < count;
       i += int64_t(gridDim.x) * blockDim.x * 4) {
    float4 v[kMaxSplits];
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s)
      if (s < n_splits) v[s] = *reinterpret_cast<const float4*>(parts + s * stride + i);
    float4 acc = v[0];
#pragma unroll
    for (int s = 1; s < kMaxSplits; ++s) {
      if (s < n_splits) {
        acc.x += v[s].x;
        acc.y += v[s].y;
        acc.z += v[s].z;
        acc.w += v[s].w;
      }
    }
    const float r[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float v = round ? bf16_round(r[c]) : r[c];
      if constexpr (std::is_same<YT, __nv_bfloat16>::value)
        y[i + c] = __float2bfloat16_rn(v);
      else
        y[i + c] = v;
    }
  }
}

struct DenseLayout {
  void *xs, *hs;
  float *xscale, *parts;
  int64_t cap;
  int max_splits;
  size_t bytes;
};

int64_t split_bound(int64_t n_tokens, int dim) {
  const int64_t units = ceil_div(dim, 128) * ceil_div(n_tokens, 128);
  return std::max<int64_t>(1, std::min<int64_t>(kMaxSplits, kSplitCtaBound / units));
}

DenseLayout dense_layout(int64_t n_tokens, int dim, int inter, void* base) {
  DenseLayout L{};
  L.cap = dsm_stage_rows_cap(n_tokens);
  L.max_splits = int(split_bound(n_tokens, dim));
  char* p = static_cast<char*>(base);
  size_t off = 0;
  auto take = [&](size_t b) {
    void* q = p ? p + off : nullptr;
    off += (b + 255) / 256 * 256;
    return q;
  };
  L.xs = take(dsm_stage_bytes(L.cap, dim));
  L.xscale = static_cast<float*>(take(size_t(L.cap) * 4));
  L.hs = take(dsm_stage_bytes(L.cap, inter));
  L.parts = static_cast<float*>(take(size_t(L.max_splits) * size_t(n_tokens) * dim * 4));
  L.bytes = off;
  return L;
}

// o[row_map[r] * ldo + c] (row_map NULL: row r) = sum over s of parts[s][r][c], in split order:
// the split-K linear's fp32 rows
__global__ void __launch_bounds__(256) sum_splits_rows_kernel(const float* __restrict__ parts, int n_splits,
                                                              int64_t n_rows, int dim, int ldo,
                                                              const int32_t* __restrict__ row_map,
                                                              float* __restrict__ o) {
  // four consecutive columns per thread: dim, ldo and the pointers are 16-byte multiples
  const int64_t count = n_rows * dim;
  for (int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < count;
       i += int64_t(gridDim.x) * blockDim.x * 4) {
    float4 v[kMaxSplits];  // every slab's load in flight before the adds, which keep split order
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s)
      if (s < n_splits) v[s] = *reinterpret_cast<const float4*>(parts + s * count + i);
    float4 acc = v[0];
#pragma unroll
    for (int s = 1; s < kMaxSplits; ++s) {
      if (s < n_splits) {
        acc.x += v[s].x;
        acc.y += v[s].y;
        acc.z += v[s].z;
        acc.w += v[s].w;
      }
    }
    const int64_t r = i / dim;
    const int c = int(i % dim);
    const int64_t orow = row_map ? int64_t(row_map[r]) : r;
    *reinterpret_cast<float4*>(o + orow * ldo + c) = acc;
  }
}

}  // namespace
}  // namespace dsm

using namespace dsm;

extern "C" size_t dsm_dense_mlp_workspace_bytes(int64_t n_tokens, int dim, int inter) {
  if (n_tokens <= 0 || dim <= 0 || inter <= 0) return 0;
  return dense_layout(n_tokens, dim, inter, nullptr).bytes;
}

extern "C" int dsm_dense_mlp(const void* x, int x_dtype, int64_t n_tokens, int dim, int inter, int wfmt,
                             int group_size, const void* w1, const void* w3, const void* w2, int act,
                             float swiglu_limit, int round_gu, int round_o, void* y, int y_dtype, void* workspace,
                             size_t workspace_bytes, void* stream) {
  DSM_REQUIRE(n_tokens >= 0 && dim > 0 && inter > 0, "dsm_dense_mlp: bad shape");
  DSM_REQUIRE(dim % 4 == 0, "dsm_dense_mlp: dim must be a multiple of 4");
  DSM_REQUIRE(x && w1 && w3 && w2 && y, "dsm_dense_mlp: null pointer");
  DSM_REQUIRE(y_dtype == DSM_DT_F32 || y_dtype == DSM_DT_BF16, "dsm_dense_mlp: y must be F32 or BF16");
  if (n_tokens == 0) return DSM_OK;
  const DenseLayout L = dense_layout(n_tokens, dim, inter, workspace);
  if (!workspace || workspace_bytes < L.bytes) return fail(DSM_ERR_WORKSPACE, "dsm_dense_mlp: workspace too small");
  cudaStream_t st = as_stream(stream);
  int rc = dsm_stage_rows(x, x_dtype, n_tokens, dim, nullptr, n_tokens, 1, L.xs, L.cap, L.xscale, stream);
  if (rc) return rc;
  const float hs = h_scale_for(act, swiglu_limit);
  rc = dsm_expert_gate_up(L.xs, L.xscale, L.cap, dim, nullptr, 1, wfmt, group_size, w1, w3, inter, act,
                          swiglu_limit, round_gu, L.hs, hs, n_tokens, stream);
  if (rc) return rc;
  int splits = 1;
  if (tm_supports(wfmt) && expert_regime() != 1)
    splits = tm_down_splits(inter, dim, n_tokens, L.max_splits);
  if (splits > 1) {
    rc = expert_tm_down_split(wfmt, group_size, L.hs, hs, L.cap, inter, w2, dim, splits, L.parts, n_tokens, stream);
  } else {
    rc = dsm_expert_down(L.hs, hs, L.cap, inter, nullptr, 1, wfmt, group_size, w2, dim, 0, L.parts, dim, nullptr,
                         n_tokens, stream);
  }
  if (rc) return rc;
  const int64_t count = n_tokens * dim;
  const int grid = int(std::min<int64_t>(ceil_div(count, 4 * 256), 4 * num_sms()));
  if (y_dtype == DSM_DT_BF16)
    reduce_splits_kernel<<<grid, 256, 0, st>>>(L.parts, splits, count, count, round_o,
                                               static_cast<__nv_bfloat16*>(y));
  else
    reduce_splits_kernel<<<grid, 256, 0, st>>>(L.parts, splits, count, count, round_o, static_cast<float*>(y));
  return check_launch("reduce_splits");
}

extern "C" size_t dsm_linear_splitk_workspace_bytes(int64_t n_rows, int out_dim) {
  if (n_rows <= 0 || out_dim <= 0) return 0;
  return size_t(kMaxSplits) * size_t(n_rows) * size_t(out_dim) * 4;
}

extern "C" int dsm_linear_splitk(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim,
                                 int wfmt, int group_size, const void* w_packed, int out_dim, float* o_rows, int ldo,
                                 int64_t n_rows, void* ws, size_t ws_bytes, void* stream) {
  DSM_REQUIRE(out_dim > 0 && k_dim > 0 && n_rows >= 0 && ldo >= out_dim, "dsm_linear_splitk: bad shape");
  DSM_REQUIRE(wfmt >= DSM_WFMT_F16 && wfmt <= DSM_WFMT_AFFINE4, "dsm_linear_splitk: unknown weight format");
  if (wfmt == DSM_WFMT_AFFINE8)
    DSM_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, "dsm_linear_splitk: affine8 group_size");
  if (wfmt == DSM_WFMT_AFFINE4)
    DSM_REQUIRE(group_size == 64 || group_size == 128, "dsm_linear_splitk: affine4 group_size");
  DSM_REQUIRE(x_staged && x_row_scale && w_packed && o_rows, "dsm_linear_splitk: NULL pointer");
  if (n_rows == 0) return DSM_OK;
  const bool aligned = (reinterpret_cast<uintptr_t>(o_rows) & 15) == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0;
  const bool can_split = ws && aligned && out_dim % 4 == 0 && ldo % 4 == 0;
  float* parts = static_cast<float*>(ws);
  int splits = 1;
  if (can_split && !tm_supports(wfmt)) {  // the streaming kernel (f16, fp8) takes its own split
    DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(n_rows), "dsm_linear_splitk: rows_cap too small");
    if (ws_bytes < dsm_linear_splitk_workspace_bytes(n_rows, out_dim))
      return fail(DSM_ERR_WORKSPACE, "dsm_linear_splitk: workspace too small");
    int rc = expert_stream_split(wfmt, group_size, x_staged, x_row_scale, rows_cap, k_dim, nullptr, 1, w_packed,
                                 out_dim, n_rows, kMaxSplits, parts, stream, &splits);
    if (rc != DSM_OK) return rc;
  } else if (can_split) {
    splits = tm_down_splits(k_dim, out_dim, n_rows, kMaxSplits);
    if (splits > 1) {
      DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(n_rows), "dsm_linear_splitk: rows_cap too small");
      const size_t need = size_t(splits) * size_t(n_rows) * size_t(out_dim) * 4;
      if (ws_bytes < need) return fail(DSM_ERR_WORKSPACE, "dsm_linear_splitk: workspace too small");
      int rc = expert_tm_down_split(wfmt, group_size, x_staged, 1.f, rows_cap, k_dim, w_packed, out_dim, splits,
                                    parts, n_rows, stream, x_row_scale);
      if (rc != DSM_OK) return rc;
    }
  }
  if (splits <= 1)
    return dsm_linear(x_staged, x_row_scale, rows_cap, k_dim, wfmt, group_size, w_packed, out_dim, o_rows, ldo,
                      n_rows, stream);
  const int64_t count = n_rows * out_dim;
  const int grid = int(std::min<int64_t>(ceil_div(count, 4 * 256), 4 * num_sms()));
  sum_splits_rows_kernel<<<grid, 256, 0, as_stream(stream)>>>(parts, splits, n_rows, out_dim, ldo, nullptr, o_rows);
  return check_launch("sum_splits_rows");
}

extern "C" int dsm_grouped_linear_splitk(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim,
                                         int wfmt, int group_size, const void* w_packed, int n_groups,
                                         const int32_t* offsets, int out_dim, float* o_rows, int ldo,
                                         const int32_t* o_row_map, int64_t n_rows, void* ws, size_t ws_bytes,
                                         void* stream) {
  DSM_REQUIRE(out_dim > 0 && k_dim > 0 && n_rows >= 0 && ldo >= out_dim && n_groups >= 1 && n_groups <= 4096,
              "dsm_grouped_linear_splitk: bad shape");
  DSM_REQUIRE(x_staged && x_row_scale && w_packed && o_rows && offsets, "dsm_grouped_linear_splitk: NULL pointer");
  if (n_rows == 0) return DSM_OK;
  const bool aligned = (reinterpret_cast<uintptr_t>(o_rows) & 15) == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0;
  int splits = 1;
  if (ws && aligned && out_dim % 4 == 0 && ldo % 4 == 0 && !tm_supports(wfmt) &&
      (wfmt == DSM_WFMT_F16 || wfmt == DSM_WFMT_FP8_B128)) {
    DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(n_rows), "dsm_grouped_linear_splitk: rows_cap too small");
    if (ws_bytes < dsm_linear_splitk_workspace_bytes(n_rows, out_dim))
      return fail(DSM_ERR_WORKSPACE, "dsm_grouped_linear_splitk: workspace too small");
    int rc = expert_stream_split(wfmt, group_size, x_staged, x_row_scale, rows_cap, k_dim, offsets, n_groups,
                                 w_packed, out_dim, n_rows, kMaxSplits, static_cast<float*>(ws), stream, &splits);
    if (rc != DSM_OK) return rc;
  }
  if (splits <= 1)
    return dsm_grouped_linear(x_staged, x_row_scale, rows_cap, k_dim, wfmt, group_size, w_packed, n_groups, offsets,
                              out_dim, o_rows, ldo, o_row_map, n_rows, stream);
  const int64_t count = n_rows * out_dim;
  const int grid = int(std::min<int64_t>(ceil_div(count, 4 * 256), 4 * num_sms()));
  sum_splits_rows_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const float*>(ws), splits, n_rows, out_dim,
                                                                ldo, o_row_map, o_rows);
  return check_launch("sum_splits_rows");
}
