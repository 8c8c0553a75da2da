// Router: Gate.__call__ of the reference (dspark_mlx/model/moe.py:62-79).
//
// Two kernels:
//   gate_logits  scores[N, E] = x_f32 . W^T, accumulated in fp64 and rounded once to fp32:
//                fp32 x fp32 products are exact in fp64, so the logit is the correctly
//                rounded dot product whatever the summation order -- top-k selection then
//                depends only on the scores, not on an accumulation order.
//   gate_topk    one warp per token: activation, top-k of (score + bias) or hash lookup,
//                gather of the unbiased scores, renormalisation, route_scale.
//
// Top-k order: ascending by biased score, the best expert in the last slot, exactly the
// order of ``argsort(scores + bias)[..., -k:]``; equal scores rank by expert id (the
// higher id ranks higher, as a stable ascending sort leaves them).
#include <cfloat>

#include "common.cuh"

namespace dsm {
namespace {

constexpr int kLT = 32;  // tokens per tile
constexpr int kLE = 32;  // experts per tile
constexpr int kLK = 32;  // K per smem stage

template <typename XT>
__global__ void __launch_bounds__(256) gate_logits_kernel(const XT* __restrict__ x, const float* __restrict__ w,
                                                          float* __restrict__ scores, int64_t n, int dim,
                                                          int n_experts) {
  __shared__ double xs[kLT][kLK + 1];
  __shared__ double ws[kLE][kLK + 1];
  const int tid = threadIdx.x;
  const int64_t t0 = int64_t(blockIdx.y) * kLT;
  const int e0 = blockIdx.x * kLE;
  // thread computes tokens (ty, ty+16) x experts (tx, tx+16)
  const int tx = tid & 15, ty = tid >> 4;
  double acc[2][2] = {{0.0, 0.0}, {0.0, 0.0}};
  for (int k0 = 0; k0 < dim; k0 += kLK) {
    for (int i = tid; i < kLT * kLK; i += 256) {
      const int r = i / kLK, c = i % kLK;
      const int64_t t = t0 + r;
      const int k = k0 + c;
      xs[r][c] = (t < n && k < dim) ? double(load_as_float(x, t * dim + k)) : 0.0;
      const int e = e0 + r;
      ws[r][c] = (e < n_experts && k < dim) ? double(w[int64_t(e) * dim + k]) : 0.0;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < kLK; ++c) {
      const double a0 = xs[ty][c], a1 = xs[ty + 16][c];
      const double b0 = ws[tx][c], b1 = ws[tx + 16][c];
      acc[0][0] = fma(a0, b0, acc[0][0]);
      acc[0][1] = fma(a0, b1, acc[0][1]);
      acc[1][0] = fma(a1, b0, acc[1][0]);
      acc[1][1] = fma(a1, b1, acc[1][1]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int64_t t = t0 + ty + 16 * i;
      const int e = e0 + tx + 16 * j;
      if (t < n && e < n_experts) scores[t * n_experts + e] = float(acc[i][j]);
    }
}

__device__ __forceinline__ float activate(float v, int score_func) {
  if (score_func == DSM_SCORE_SIGMOID) return 1.f / (1.f + expf(-v));
  // sqrt(softplus(v)), softplus = max(v,0) + log1p(exp(-|v|))  (moe.py:31-34)
  return sqrtf(fmaxf(v, 0.f) + log1pf(expf(-fabsf(v))));
}

// (value, index) ordering: larger value wins; on equal values the larger index wins.
__device__ __forceinline__ bool beats(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i > bi);
}

constexpr int kMaxExpertsPerLane = 32;  // E <= 1024

template <typename IDT>
__global__ void __launch_bounds__(128) gate_topk_kernel(const float* __restrict__ scores, int64_t n,
                                                        int n_experts, const float* __restrict__ bias,
                                                        const int32_t* __restrict__ tid2eid, int64_t vocab,
                                                        const IDT* __restrict__ ids, int64_t n_ids, int topk,
                                                        int score_func, float route_scale,
                                                        float* __restrict__ weights_out,
                                                        int32_t* __restrict__ idx_out) {
  const int lane = threadIdx.x & 31;
  const int64_t t = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (t >= n) return;
  const float* row = scores + t * n_experts;
  const int per_lane = (n_experts + 31) / 32;
  float act[kMaxExpertsPerLane];  // unbiased activated scores
  float sel[kMaxExpertsPerLane];  // selection keys (score + bias)
  // softmax needs the row max and sum first
  float mx = -FLT_MAX, sum = 0.f;
  if (score_func == DSM_SCORE_SOFTMAX) {
    for (int j = 0; j < per_lane; ++j) {
      const int e = lane + 32 * j;
      if (e < n_experts) mx = fmaxf(mx, row[e]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int j = 0; j < per_lane; ++j) {
      const int e = lane + 32 * j;
      if (e < n_experts) sum += expf(row[e] - mx);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
#pragma unroll
  for (int j = 0; j < kMaxExpertsPerLane; ++j) {
    const int e = lane + 32 * j;
    float a = -FLT_MAX, s = -FLT_MAX;
    if (j < per_lane && e < n_experts) {
      const float v = row[e];
      a = score_func == DSM_SCORE_SOFTMAX ? expf(v - mx) / sum : activate(v, score_func);
      s = bias ? a + bias[e] : a;
    }
    act[j] = a;
    sel[j] = s;
  }
  float wsel[16];
  int isel[16];
  if (tid2eid) {
    // hash mode (moe.py:71-72): the ids broadcast against the tokens (length N or 1)
    const int64_t id = static_cast<int64_t>(ids[n_ids == 1 ? 0 : t]);
    const bool ok = id >= 0 && id < vocab;
    if (!ok && lane == 0) raise_device_error(DSM_DEV_ERR_TOKEN_RANGE);
    for (int s = 0; s < topk; ++s) {
      int e = ok ? tid2eid[id * topk + s] : 0;
      if (e < 0 || e >= n_experts) {
        if (lane == 0) raise_device_error(DSM_DEV_ERR_EXPERT_RANGE);
        e = 0;
      }
      // fetch act[e] from its owner lane
      float v = -FLT_MAX;
#pragma unroll
      for (int j = 0; j < kMaxExpertsPerLane; ++j)
        if (j == (e >> 5)) v = act[j];
      isel[s] = e;
      wsel[s] = __shfl_sync(0xffffffffu, v, e & 31);
    }
  } else {
    // k rounds of arg-max over (key, index); write from the last slot down (ascending order)
    for (int s = topk - 1; s >= 0; --s) {
      float bv = -INFINITY, ba = 0.f;
      int bi = -1;
#pragma unroll
      for (int j = 0; j < kMaxExpertsPerLane; ++j) {
        const int e = lane + 32 * j;
        if (j < per_lane && e < n_experts && beats(sel[j], e, bv, bi)) {
          bv = sel[j];
          bi = e;
          ba = act[j];
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const float oa = __shfl_xor_sync(0xffffffffu, ba, o);
        if (beats(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
          ba = oa;
        }
      }
      // remove the winner
      if ((bi & 31) == lane) {
#pragma unroll
        for (int j = 0; j < kMaxExpertsPerLane; ++j)
          if (j == (bi >> 5)) sel[j] = -INFINITY;
      }
      isel[s] = bi;
      wsel[s] = ba;
    }
  }
  if (lane == 0) {
    float denom = 0.f;
    if (score_func != DSM_SCORE_SOFTMAX)
      for (int s = 0; s < topk; ++s) denom += wsel[s];
    for (int s = 0; s < topk; ++s) {
      float v = wsel[s];
      if (score_func != DSM_SCORE_SOFTMAX) v = v / denom;
      weights_out[t * topk + s] = v * route_scale;
      idx_out[t * topk + s] = isel[s];
    }
  }
}

}  // namespace
}  // namespace dsm

extern "C" int dsm_router(const void* x, int x_dtype, int64_t n_tokens, int dim, const float* gate_weight,
                          int n_experts, const float* gate_bias, const int32_t* tid2eid, int64_t vocab,
                          const void* input_ids, int ids_dtype, int64_t n_ids, int topk, int score_func,
                          float route_scale, float* scores_ws, float* weights_out, int32_t* indices_out,
                          void* stream) {
  using namespace dsm;
  DSM_REQUIRE(n_tokens >= 0 && dim > 0 && n_experts > 0, "dsm_router: bad shape");
  DSM_REQUIRE(n_experts <= 32 * kMaxExpertsPerLane, "dsm_router: n_experts > 1024 unsupported");
  DSM_REQUIRE(topk >= 1 && topk <= 16 && topk <= n_experts, "dsm_router: topk must be in [1, min(16, E)]");
  DSM_REQUIRE(x_dtype == DSM_DT_F32 || x_dtype == DSM_DT_BF16, "dsm_router: x must be F32 or BF16");
  DSM_REQUIRE(score_func >= DSM_SCORE_SOFTMAX && score_func <= DSM_SCORE_SQRTSOFTPLUS, "dsm_router: bad score_func");
  DSM_REQUIRE(x && gate_weight && scores_ws && weights_out && indices_out, "dsm_router: NULL pointer");
  if (tid2eid) {
    DSM_REQUIRE(input_ids != nullptr, "dsm_router: hash routing needs input_ids");
    DSM_REQUIRE(ids_dtype == DSM_DT_I32 || ids_dtype == DSM_DT_I64, "dsm_router: ids must be I32 or I64");
    DSM_REQUIRE(n_ids == n_tokens || n_ids == 1,
                "dsm_router: input_ids must have one id per token or a single id (draft-block anchor)");
    DSM_REQUIRE(vocab > 0, "dsm_router: vocab must be positive");
  } else {
    DSM_REQUIRE(gate_bias != nullptr, "dsm_router: score routing needs gate_bias");
  }
  if (n_tokens == 0) return DSM_OK;
  cudaStream_t s = as_stream(stream);
  dim3 grid(unsigned(ceil_div(n_experts, kLE)), unsigned(ceil_div(n_tokens, kLT)));
  if (x_dtype == DSM_DT_BF16)
    gate_logits_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), gate_weight,
                                                           scores_ws, n_tokens, dim, n_experts);
  else
    gate_logits_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), gate_weight, scores_ws, n_tokens,
                                                   dim, n_experts);
  if (int rc = check_launch("gate_logits")) return rc;
  const unsigned blocks = unsigned(ceil_div(n_tokens, 4));
  if (ids_dtype == DSM_DT_I64 && tid2eid)
    gate_topk_kernel<int64_t><<<blocks, 128, 0, s>>>(scores_ws, n_tokens, n_experts, gate_bias, tid2eid, vocab,
                                                     static_cast<const int64_t*>(input_ids), n_ids, topk, score_func,
                                                     route_scale, weights_out, indices_out);
  else
    gate_topk_kernel<int32_t><<<blocks, 128, 0, s>>>(scores_ws, n_tokens, n_experts, gate_bias, tid2eid, vocab,
                                                     static_cast<const int32_t*>(input_ids), n_ids, topk, score_func,
                                                     route_scale, weights_out, indices_out);
  return check_launch("gate_topk");
}
