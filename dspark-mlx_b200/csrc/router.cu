// Router: Gate.__call__ of the reference (dspark_mlx/model/moe.py:62-79).
//
// Three kernels:
//   gate_partial  fp64 partial logits x_f32 . W^T over K slices on the fp64 tensor cores
//                 (mma.m8n8k4.f64). fp32 x fp32 products are exact in fp64, so every logit
//                 is the correctly rounded dot product up to fp64 summation error (~1e-16
//                 relative) whatever the summation order: top-k selection depends only on
//                 the scores, not on an accumulation order.
//   gate_reduce   sums the slices in a fixed order and rounds once to fp32.
//   gate_topk     one warp per token: activation, top-k of (score + bias) or hash lookup,
//                 gather of the unbiased scores, renormalisation, route_scale.
//
// Top-k order: ascending by biased score, the best expert in the last slot, exactly the
// order of ``argsort(scores + bias)[..., -k:]``; equal scores rank by expert id (the
// higher id ranks higher, as a stable ascending sort leaves them).
#include <cfloat>
#include <type_traits>

#include "common.cuh"

namespace dsm {
namespace {

// CTA tiles: PT tokens x PE experts x one K slice, in PKS-wide K sub-chunks; 8 warps in a
// 4 x 2 grid, each (PT / 4) tokens x (PE / 2) experts of m8n8 tiles. Decode-sized calls take
// 64 x 32 (32-wide sub-chunks, 16 x 16 per warp: little padding at 56-448 tokens); from
// kWideTokens tokens, 128 x 64 (16-wide sub-chunks, 32 x 32 per warp: each fragment load
// feeds twice the MMAs). Shared pitch PKS + 4 doubles (4 mod 16) makes the m8n8k4 fragment
// loads (8 rows x 4 consecutive K) conflict-free.
constexpr int64_t kWideTokens = 1024;
template <int PT>
struct RouterTile {
  static constexpr int PE = PT == 128 ? 64 : 32;
  static constexpr int PKS = PT == 128 ? 16 : 32;
  static constexpr int kPitch = PKS + 4;
  static constexpr int TI = PT / 4 / 8, TJ = PE / 2 / 8;  // m8n8 tiles per warp
  static_assert(PT * PKS == 256 * 8 && PE * PKS == 256 * 4, "one 8-value x load and one 4-value w load per thread");
};
inline int router_tile_tokens(int64_t n_tokens) { return n_tokens >= kWideTokens ? 128 : 64; }

__device__ __forceinline__ void dmma(double (&d)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
               : "+d"(d[0]), "+d"(d[1])
               : "d"(a), "d"(b));
}

// K slice of one partial-logit CTA. Decode-sized batches use 256. Larger batches split K
// until the grid reaches ~2 CTAs per SM of a B200 (a fixed target, so the workspace query
// and the launch agree on every device), with slices of at least 256; from ~2 000 tokens K
// stays whole. The fp64 partials are summed in a fixed order: the logits do not depend on
// the split beyond fp64 rounding.
int router_k_slice(int64_t n_tokens, int dim, int n_experts) {
  if (n_tokens <= 256) return 256;
  constexpr int64_t kTargetCtas = 2 * 148;
  const int pt = router_tile_tokens(n_tokens), pe = pt == 128 ? 64 : 32;
  const int64_t tiles = ceil_div(int64_t(n_experts), int64_t(pe)) * ceil_div(n_tokens, int64_t(pt));
  int64_t slices = std::max<int64_t>(1, ceil_div(kTargetCtas, tiles));
  slices = std::min<int64_t>(slices, std::max<int64_t>(1, dim / 256));
  return int(ceil_div(ceil_div(int64_t(dim), slices), int64_t(32)) * 32);
}

template <typename XT, int PT>
__global__ void __launch_bounds__(256) gate_partial_kernel(const XT* __restrict__ x, const float* __restrict__ w,
                                                           double* __restrict__ part, int64_t n, int dim,
                                                           int n_experts, int k_slice, int vec_ok) {
  using T = RouterTile<PT>;
  constexpr int PE = T::PE, PKS = T::PKS, TI = T::TI, TJ = T::TJ;
  __shared__ double xs[PT][T::kPitch];
  __shared__ double ws[PE][T::kPitch];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int e0 = blockIdx.x * PE;
  const int ks = blockIdx.y;
  const int64_t t0 = int64_t(blockIdx.z) * PT;
  const int kbeg = ks * k_slice, kend = min(dim, kbeg + k_slice);
  const int tw = (warp & 3) * (PT / 4), ew = (warp >> 2) * (PE / 2);
  double acc[TI][TJ][2] = {};
  // each thread stages 8 x values and 4 w values per sub-chunk; the next sub-chunk's global
  // loads are issued before the current one is multiplied
  const int xr = tid / (PKS / 8), xc = (tid % (PKS / 8)) * 8;
  const int wr = tid / (PKS / 4), wc = (tid % (PKS / 4)) * 4;
  float xv[8], wv[4];
  auto fetch = [&](int k0) {
    const int64_t t = t0 + xr;
    const int k = k0 + xc;
    if (vec_ok && t < n && k + 8 <= kend) {
      if constexpr (sizeof(XT) == 2) {
        const uint4 u = *reinterpret_cast<const uint4*>(x + t * dim + k);
        const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xv[2 * i] = __uint_as_float(wd[i] << 16);
          xv[2 * i + 1] = __uint_as_float(wd[i] & 0xFFFF0000u);
        }
      } else {
        const float4 p = *reinterpret_cast<const float4*>(x + t * dim + k);
        const float4 q = *reinterpret_cast<const float4*>(x + t * dim + k + 4);
        xv[0] = p.x, xv[1] = p.y, xv[2] = p.z, xv[3] = p.w, xv[4] = q.x, xv[5] = q.y, xv[6] = q.z, xv[7] = q.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[i] = (t < n && k + i < kend) ? load_as_float(x, t * dim + k + i) : 0.f;
    }
    const int e = e0 + wr;
    const int kw = k0 + wc;
    if (vec_ok && e < n_experts && kw + 4 <= kend) {
      const float4 p = *reinterpret_cast<const float4*>(w + int64_t(e) * dim + kw);
      wv[0] = p.x, wv[1] = p.y, wv[2] = p.z, wv[3] = p.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) wv[i] = (e < n_experts && kw + i < kend) ? w[int64_t(e) * dim + kw + i] : 0.f;
    }
  };
  fetch(kbeg);
  for (int k0 = kbeg; k0 < kend; k0 += PKS) {
#pragma unroll
    for (int i = 0; i < 8; ++i) xs[xr][xc + i] = double(xv[i]);
#pragma unroll
    for (int i = 0; i < 4; ++i) ws[wr][wc + i] = double(wv[i]);
    __syncthreads();
    if (k0 + PKS < kend) fetch(k0 + PKS);
#pragma unroll
    for (int kk = 0; kk < PKS / 4; ++kk) {
      const int kc = kk * 4 + (lane & 3);
      double a[TI], b[TJ];
#pragma unroll
      for (int i = 0; i < TI; ++i) a[i] = xs[tw + 8 * i + (lane >> 2)][kc];
#pragma unroll
      for (int j = 0; j < TJ; ++j) b[j] = ws[ew + 8 * j + (lane >> 2)][kc];
#pragma unroll
      for (int i = 0; i < TI; ++i)
#pragma unroll
        for (int j = 0; j < TJ; ++j) dmma(acc[i][j], a[i], b[j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < TI; ++i)
#pragma unroll
    for (int j = 0; j < TJ; ++j)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int64_t t = t0 + tw + 8 * i + (lane >> 2);
        const int e = e0 + ew + 8 * j + (lane & 3) * 2 + c;
        if (t < n && e < n_experts) part[(int64_t(ks) * n + t) * n_experts + e] = acc[i][j][c];
      }
}

// logits[i] = fp32(sum over slices, in slice order)
__global__ void __launch_bounds__(256) gate_reduce_kernel(const double* __restrict__ part, int n_slices,
                                                          int64_t count, float* __restrict__ logits) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= count) return;
  double v = 0.0;
#pragma unroll 16
  for (int ks = 0; ks < n_slices; ++ks) v += part[int64_t(ks) * count + i];
  logits[i] = float(v);
}

__device__ __forceinline__ float activate(float v, int score_func) {
  if (score_func == DSM_SCORE_SIGMOID) return 1.f / (1.f + expf(-v));
  // sqrt(softplus(v)), softplus = max(v,0) + log1p(exp(-|v|))  (moe.py:31-34)
  return sqrtf(fmaxf(v, 0.f) + log1pf(expf(-fabsf(v))));
}

// Selection key: the biased score's bits mapped to an order-preserving unsigned (larger
// score -> larger key), expert id in the low word so that equal scores rank by expert id
// (the higher id wins, as a stable ascending sort leaves them). 0 marks a removed or absent
// expert; NaN scores map above +inf and are never produced by the supported activations.
__device__ __forceinline__ uint64_t sel_key(float v, int e) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (uint64_t(b) << 32) | uint32_t(e);
}

constexpr int kMaxExpertsPerLane = 32;  // E <= 1024

// One warp per token; PL = experts per lane (expert e = lane + 32 j).
template <typename IDT, int PL>
__global__ void __launch_bounds__(128) gate_topk_kernel(const float* __restrict__ logits, int64_t n, int n_experts,
                                                        const float* __restrict__ bias,
                                                        const int32_t* __restrict__ tid2eid, int64_t vocab,
                                                        const IDT* __restrict__ ids, int64_t n_ids, int topk,
                                                        int score_func, float route_scale,
                                                        float* __restrict__ weights_out,
                                                        int32_t* __restrict__ idx_out) {
  const int lane = threadIdx.x & 31;
  const int64_t t = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (t >= n) return;
  float act[PL];
  uint64_t key[PL];
#pragma unroll
  for (int j = 0; j < PL; ++j) {
    const int e = lane + 32 * j;
    act[j] = e < n_experts ? logits[t * n_experts + e] : -FLT_MAX;
  }
  if (score_func == DSM_SCORE_SOFTMAX) {
    float mx = -FLT_MAX, sum = 0.f;
#pragma unroll
    for (int j = 0; j < PL; ++j)
      if (lane + 32 * j < n_experts) mx = fmaxf(mx, act[j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll
    for (int j = 0; j < PL; ++j)
      if (lane + 32 * j < n_experts) sum += expf(act[j] - mx);
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int j = 0; j < PL; ++j)
      if (lane + 32 * j < n_experts) act[j] = expf(act[j] - mx) / sum;
  } else {
#pragma unroll
    for (int j = 0; j < PL; ++j)
      if (lane + 32 * j < n_experts) act[j] = activate(act[j], score_func);
  }
#pragma unroll
  for (int j = 0; j < PL; ++j) {
    const int e = lane + 32 * j;
    key[j] = e < n_experts ? sel_key(bias ? act[j] + bias[e] : act[j], e) : 0ull;
  }
  float wsel = 0.f;  // lane s (< topk) ends up holding slot s
  int isel = 0;
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
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < PL; ++j)
        if (j == (e >> 5)) v = act[j];
      v = __shfl_sync(0xffffffffu, v, e & 31);
      if (lane == s) {
        wsel = v;
        isel = e;
      }
    }
  } else {
    // k rounds of a warp-wide max over the keys; slots fill from the last one down
    for (int s = topk - 1; s >= 0; --s) {
      uint64_t best = key[0];
#pragma unroll
      for (int j = 1; j < PL; ++j) best = key[j] > best ? key[j] : best;
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      const int e = int(uint32_t(best));
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < PL; ++j)
        if (lane + 32 * j == e) {
          v = act[j];
          key[j] = 0ull;
        }
      v = __shfl_sync(0xffffffffu, v, e & 31);
      if (lane == s) {
        wsel = v;
        isel = e;
      }
    }
  }
  // renormalise over the k slots in slot order (lane s holds slot s)
  float denom = 0.f;
  if (score_func != DSM_SCORE_SOFTMAX)
    for (int s = 0; s < topk; ++s) denom += __shfl_sync(0xffffffffu, wsel, s);
  if (lane < topk) {
    const float v = score_func != DSM_SCORE_SOFTMAX ? wsel / denom : wsel;
    weights_out[t * topk + lane] = v * route_scale;
    idx_out[t * topk + lane] = isel;
  }
}

}  // namespace
}  // namespace dsm

extern "C" size_t dsm_router_workspace_bytes(int64_t n_tokens, int dim, int n_experts) {
  if (n_tokens <= 0 || dim <= 0 || n_experts <= 0) return 256;
  const int64_t slices = dsm::ceil_div(dim, dsm::router_k_slice(n_tokens, dim, n_experts));
  const size_t cells = size_t(n_tokens) * size_t(n_experts);
  return cells * (size_t(slices) * sizeof(double) + sizeof(float));
}

extern "C" int dsm_router(const void* x, int x_dtype, int64_t n_tokens, int dim, const float* gate_weight,
                          int n_experts, const float* gate_bias, const int32_t* tid2eid, int64_t vocab,
                          const void* input_ids, int ids_dtype, int64_t n_ids, int topk, int score_func,
                          float route_scale, void* workspace, float* weights_out, int32_t* indices_out,
                          void* stream) {
  using namespace dsm;
  DSM_REQUIRE(n_tokens >= 0 && dim > 0 && n_experts > 0, "dsm_router: bad shape");
  DSM_REQUIRE(n_experts <= 32 * kMaxExpertsPerLane, "dsm_router: n_experts > 1024 unsupported");
  DSM_REQUIRE(topk >= 1 && topk <= 32 && topk <= n_experts, "dsm_router: topk must be in [1, min(32, E)]");
  DSM_REQUIRE(x_dtype == DSM_DT_F32 || x_dtype == DSM_DT_BF16, "dsm_router: x must be F32 or BF16");
  DSM_REQUIRE(score_func >= DSM_SCORE_SOFTMAX && score_func <= DSM_SCORE_SQRTSOFTPLUS, "dsm_router: bad score_func");
  DSM_REQUIRE(x && gate_weight && workspace && weights_out && indices_out, "dsm_router: NULL pointer");
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
  const int k_slice = router_k_slice(n_tokens, dim, n_experts);
  const int n_slices = int(ceil_div(dim, k_slice));
  double* part = static_cast<double*>(workspace);
  float* logits = reinterpret_cast<float*>(part + int64_t(n_slices) * n_tokens * n_experts);
  const int vec_ok = (dim % 8 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(gate_weight) & 15) == 0);
  auto partial = [&](auto tile) {
    constexpr int PT = decltype(tile)::value;
    dim3 grid(unsigned(ceil_div(n_experts, RouterTile<PT>::PE)), unsigned(n_slices), unsigned(ceil_div(n_tokens, PT)));
    if (x_dtype == DSM_DT_BF16)
      gate_partial_kernel<__nv_bfloat16, PT><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), gate_weight,
                                                                  part, n_tokens, dim, n_experts, k_slice, vec_ok);
    else
      gate_partial_kernel<float, PT><<<grid, 256, 0, s>>>(static_cast<const float*>(x), gate_weight, part, n_tokens,
                                                          dim, n_experts, k_slice, vec_ok);
  };
  if (router_tile_tokens(n_tokens) == 128)
    partial(std::integral_constant<int, 128>{});
  else
    partial(std::integral_constant<int, 64>{});
  if (int rc = check_launch("gate_partial")) return rc;
  const int64_t count = n_tokens * n_experts;
  gate_reduce_kernel<<<unsigned(ceil_div(count, 256)), 256, 0, s>>>(part, n_slices, count, logits);
  if (int rc = check_launch("gate_reduce")) return rc;
  const unsigned blocks = unsigned(ceil_div(n_tokens, 4));
  const int pl = int(ceil_div(n_experts, 32));
#define DSM_TOPK(IDT, PL)                                                                                         \
  gate_topk_kernel<IDT, PL><<<blocks, 128, 0, s>>>(logits, n_tokens, n_experts, gate_bias, tid2eid, vocab,         \
                                                   static_cast<const IDT*>(input_ids), n_ids, topk, score_func, \
                                                   route_scale, weights_out, indices_out)
#define DSM_TOPK_PL(IDT)           \
  if (pl <= 1) DSM_TOPK(IDT, 1);   \
  else if (pl <= 2) DSM_TOPK(IDT, 2); \
  else if (pl <= 4) DSM_TOPK(IDT, 4); \
  else if (pl <= 8) DSM_TOPK(IDT, 8); \
  else if (pl <= 16) DSM_TOPK(IDT, 16); \
  else DSM_TOPK(IDT, 32);
  if (ids_dtype == DSM_DT_I64 && tid2eid) {
    DSM_TOPK_PL(int64_t)
  } else {
    DSM_TOPK_PL(int32_t)
  }
#undef DSM_TOPK_PL
#undef DSM_TOPK
  return check_launch("gate_topk");
}
