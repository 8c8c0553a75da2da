// The MoE's neighbours in the DSpark draft block (dspark_mlx/model/block.py:83-86): the
// hyper-connection reduction before the FFN and its RMSNorm, and the re-expansion after it.
//
//   dsm_hc_pre_norm  hc_pre (dspark_mlx/model/hyper.py:24-42, with kernels.hc_split_sinkhorn,
//                    kernels.py:60-85) followed by ffn_norm (RMSNorm, model/norm_rope.py:22-39):
//                    x [n, hc, d] -> the MoE input [n, d], plus post [n, hc], comb [n, hc, hc]
//   dsm_hc_post      hc_post (hyper.py:45-51): out[c] = post[c] * h + sum_a comb[a, c] * res[a]
//   dsm_hc_head_norm hc_head (hyper.py:52-67) and the draft head's final RMSNorm
//                    (block.py:111-112): x [n, hc, d] -> y [n, d], RMSNorm(y) [n, d] and the
//                    hidden half of the confidence projection (heads.py:46-48)
//
// Everything is fp32 inside, cast to the activation dtype where the reference casts. One
// CTA per token for the pre-norm: a single pass over the token's hc*d values accumulates the
// sum of squares and the (2 + hc) * hc mix projections (the projection matrix stays in L2
// across tokens), a block reduction, the Sinkhorn split on one thread, then the pre-weighted
// sum of the copies (rounded to the activation dtype, kept in shared memory) and its RMS.
#include "common.cuh"

namespace dsm {
namespace {

constexpr int kHcThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float sigmoid_f(float v) { return 1.f / (1.f + expf(-v)); }

// block-wide sum of NV values per thread (in place: every thread gets the totals)
template <int NV>
__device__ __forceinline__ void block_sum(float (&v)[NV], float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int o = 16; o; o >>= 1) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
  __syncthreads();
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < NV; ++i) red[warp * NV + i] = v[i];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float s = 0.f;
    for (int w = 0; w < kHcThreads / 32; ++w) s += red[w * NV + i];
    v[i] = s;
  }
}

// PAIR: the token's pass 1 split between the two CTAs of a cluster, each over half of the
// hc * dim columns (each reads half of the projection rows from L2). CTA 1 stores its sums
// into CTA 0's shared memory (distributed shared memory), CTA 0 adds them after its own and
// finishes the token alone.
template <typename T, int HC, bool PAIR>
__device__ __forceinline__ void hc_pre_norm_body(const T* __restrict__ x, int dim, const float* __restrict__ fn,
                                                 const float* __restrict__ scale, const float* __restrict__ base,
                                                 int iters, float norm_eps, float hc_eps,
                                                 const float* __restrict__ weight, T* __restrict__ xn,
                                                 float* __restrict__ post_out, float* __restrict__ comb_out) {
  constexpr int MIX = (2 + HC) * HC;
  extern __shared__ float ysm[];  // dim floats: the reduced row, rounded to T
  __shared__ float red[(kHcThreads / 32) * (MIX + 1)];
  __shared__ float pre_s[HC];
  __shared__ float peer_acc[MIX + 1];  // PAIR: CTA 1's sums, written by CTA 1 into CTA 0
  uint32_t rank = 0;
  if constexpr (PAIR) asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int64_t t = PAIR ? int64_t(blockIdx.x >> 1) : int64_t(blockIdx.x);
  const int hcd = HC * dim;
  const T* xt = x + t * hcd;
  // this CTA's columns: all of them, or half (hcd is even: dim is)
  const int k_lo = PAIR ? int(rank) * (hcd / 2) : 0, k_hi = PAIR ? k_lo + hcd / 2 : hcd;

  // pass 1: sum of squares and the mix projections of the flattened copies
  float acc[MIX + 1];
#pragma unroll
  for (int i = 0; i <= MIX; ++i) acc[i] = 0.f;
  // kU of the thread's columns per step: all their loads (x and the MIX projection rows,
  // which stay in L2 across tokens) are issued before the multiply-adds, so a step waits on
  // one L2 round trip instead of kU; the adds keep the thread's column order.
  constexpr int kU = 4;
  int k = k_lo + int(threadIdx.x);
  for (; k + (kU - 1) * kHcThreads < k_hi; k += kU * kHcThreads) {
    float v[kU], f[kU][MIX];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int ku = k + u * kHcThreads;
      v[u] = to_f(xt[ku]);
#pragma unroll
      for (int j = 0; j < MIX; ++j) f[u][j] = fn[int64_t(j) * hcd + ku];
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      acc[MIX] = fmaf(v[u], v[u], acc[MIX]);
#pragma unroll
      for (int j = 0; j < MIX; ++j) acc[j] = fmaf(v[u], f[u][j], acc[j]);
    }
  }
  for (; k < k_hi; k += kHcThreads) {
    const float v = to_f(xt[k]);
    acc[MIX] = fmaf(v, v, acc[MIX]);
#pragma unroll
    for (int j = 0; j < MIX; ++j) acc[j] = fmaf(v, fn[int64_t(j) * hcd + k], acc[j]);
  }
  block_sum(acc, red);
  if constexpr (PAIR) {
    if (rank == 1 && int(threadIdx.x) <= MIX) {  // this half's sums into CTA 0's peer_acc
      uint32_t dst;
      asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(dst) : "r"(smem_u32(&peer_acc[threadIdx.x])));
      float mine = 0.f;
#pragma unroll
      for (int i = 0; i <= MIX; ++i)
        if (i == int(threadIdx.x)) mine = acc[i];
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(mine) : "memory");
    }
    // every thread of both CTAs: CTA 1's stores are visible in CTA 0 after this barrier
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (rank == 1) return;
#pragma unroll
    for (int i = 0; i <= MIX; ++i) acc[i] += peer_acc[i];  // first half, then second
  }

  if (threadIdx.x == 0) {  // hc_split_sinkhorn on the token's mixes
    const float inv_rms = rsqrtf(acc[MIX] / float(hcd) + norm_eps);
    float m[MIX];
#pragma unroll
    for (int j = 0; j < MIX; ++j) m[j] = acc[j] * inv_rms;
#pragma unroll
    for (int c = 0; c < HC; ++c) {
      pre_s[c] = sigmoid_f(m[c] * scale[0] + base[c]) + hc_eps;
      post_out[t * HC + c] = 2.f * sigmoid_f(m[HC + c] * scale[1] + base[HC + c]);
    }
    float cb[HC][HC];
#pragma unroll
    for (int a = 0; a < HC; ++a) {  // row softmax
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        cb[a][c] = m[2 * HC + a * HC + c] * scale[2] + base[2 * HC + a * HC + c];
        mx = fmaxf(mx, cb[a][c]);
      }
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        cb[a][c] = expf(cb[a][c] - mx);
        s += cb[a][c];
      }
#pragma unroll
      for (int c = 0; c < HC; ++c) cb[a][c] = cb[a][c] / s + hc_eps;
    }
    auto col_norm = [&]() {
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        float s = 0.f;
#pragma unroll
        for (int a = 0; a < HC; ++a) s += cb[a][c];
        s += hc_eps;
#pragma unroll
        for (int a = 0; a < HC; ++a) cb[a][c] /= s;
      }
    };
    col_norm();
    for (int it = 1; it < iters; ++it) {
#pragma unroll
      for (int a = 0; a < HC; ++a) {  // row normalisation
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < HC; ++c) s += cb[a][c];
        s += hc_eps;
#pragma unroll
        for (int c = 0; c < HC; ++c) cb[a][c] /= s;
      }
      col_norm();
    }
#pragma unroll
    for (int a = 0; a < HC; ++a)
#pragma unroll
      for (int c = 0; c < HC; ++c) comb_out[(t * HC + a) * HC + c] = cb[a][c];
  }
  __syncthreads();

  // pass 2: y = sum_c pre[c] * x[c] (cast to T), then RMSNorm(y) * weight (cast to T)
  float sq[1] = {0.f};
  for (int j = threadIdx.x; j < dim; j += kHcThreads) {
    float y = 0.f;
#pragma unroll
    for (int c = 0; c < HC; ++c) y = __fadd_rn(y, __fmul_rn(pre_s[c], to_f(xt[c * dim + j])));  // products, then sum
    const float yq = to_f(from_f<T>(y));
    ysm[j] = yq;
    sq[0] = fmaf(yq, yq, sq[0]);
  }
  block_sum(sq, red);
  const float r = rsqrtf(sq[0] / float(dim) + norm_eps);
  T* out = xn + t * dim;
  for (int j = threadIdx.x; j < dim; j += kHcThreads) {
    const float v = ysm[j] * r;
    out[j] = from_f<T>(weight ? weight[j] * v : v);
  }
}

template <typename T, int HC>
__global__ void __launch_bounds__(kHcThreads) hc_pre_norm_kernel(const T* __restrict__ x, int dim,
                                                                   const float* __restrict__ fn,
                                                                   const float* __restrict__ scale,
                                                                   const float* __restrict__ base, int iters,
                                                                   float norm_eps, float hc_eps,
                                                                   const float* __restrict__ weight, T* __restrict__ xn,
                                                                   float* __restrict__ post_out,
                                                                   float* __restrict__ comb_out) {
  hc_pre_norm_body<T, HC, false>(x, dim, fn, scale, base, iters, norm_eps, hc_eps, weight, xn, post_out, comb_out);
}

// two CTAs per token (grid 2 n, clusters of 2): few tokens, whose CTAs alone would leave most
// SMs idle while each reads all (2 + hc) * hc projection rows
template <typename T, int HC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kHcThreads)
    hc_pre_norm_pair_kernel(const T* __restrict__ x, int dim, const float* __restrict__ fn,
                            const float* __restrict__ scale, const float* __restrict__ base, int iters, float norm_eps,
                            float hc_eps, const float* __restrict__ weight, T* __restrict__ xn,
                            float* __restrict__ post_out, float* __restrict__ comb_out) {
  hc_pre_norm_body<T, HC, true>(x, dim, fn, scale, base, iters, norm_eps, hc_eps, weight, xn, post_out, comb_out);
}

template <typename T, int HC>
__global__ void __launch_bounds__(kHcThreads) hc_post_kernel(const T* __restrict__ h, const T* __restrict__ res,
                                                               int dim, const float* __restrict__ post,
                                                               const float* __restrict__ comb, T* __restrict__ out) {
  const int64_t t = blockIdx.y;
  const int j = blockIdx.x * kHcThreads + threadIdx.x;
  if (j >= dim) return;
  float p[HC], cm[HC][HC], r[HC];
#pragma unroll
  for (int c = 0; c < HC; ++c) p[c] = post[t * HC + c];
#pragma unroll
  for (int a = 0; a < HC; ++a) {
    r[a] = to_f(res[(t * HC + a) * dim + j]);
#pragma unroll
    for (int c = 0; c < HC; ++c) cm[a][c] = comb[(t * HC + a) * HC + c];
  }
  const float hv = to_f(h[t * dim + j]);
#pragma unroll
  for (int c = 0; c < HC; ++c) {
    float s = 0.f;
#pragma unroll
    for (int a = 0; a < HC; ++a) s = __fadd_rn(s, __fmul_rn(cm[a][c], r[a]));
    out[(t * HC + c) * dim + j] = from_f<T>(__fadd_rn(__fmul_rn(p[c], hv), s));
  }
}

// hc_head (hyper.py:52-67) then the final RMSNorm: y = sum_c pre[c] x[c] with
// pre = sigmoid(mixes * scale + base) + hc_eps, mixes = (x . fn) * rsqrt(mean(x^2) + eps); y
// is rounded to T and written out; xn = RMSNorm(y) * weight, rounded to T; and
// conf[t] = sum_j y[j] * conf_w[j] (the hidden half of the confidence projection).
template <typename T, int HC>
__global__ void __launch_bounds__(kHcThreads) hc_head_norm_kernel(const T* __restrict__ x, int dim,
                                                                    const float* __restrict__ fn,
                                                                    const float* __restrict__ scale,
                                                                    const float* __restrict__ base, float norm_eps,
                                                                    float hc_eps, const float* __restrict__ weight,
                                                                    const float* __restrict__ conf_w,
                                                                    T* __restrict__ y_out, T* __restrict__ xn,
                                                                    float* __restrict__ conf_out) {
  extern __shared__ float ysm[];  // dim floats: the reduced row, rounded to T
  __shared__ float red[(kHcThreads / 32) * (HC + 2)];
  __shared__ float pre_s[HC];
  const int64_t t = blockIdx.x;
  const int hcd = HC * dim;
  const T* xt = x + t * hcd;
  float acc[HC + 1];
#pragma unroll
  for (int i = 0; i <= HC; ++i) acc[i] = 0.f;
  // as in hc_pre_norm_kernel: kU columns' loads in flight per step, adds in column order
  constexpr int kU = 8;
  int k = threadIdx.x;
  for (; k + (kU - 1) * kHcThreads < hcd; k += kU * kHcThreads) {
    float v[kU], f[kU][HC];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int ku = k + u * kHcThreads;
      v[u] = to_f(xt[ku]);
#pragma unroll
      for (int j = 0; j < HC; ++j) f[u][j] = fn[int64_t(j) * hcd + ku];
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      acc[HC] = fmaf(v[u], v[u], acc[HC]);
#pragma unroll
      for (int j = 0; j < HC; ++j) acc[j] = fmaf(v[u], f[u][j], acc[j]);
    }
  }
  for (; k < hcd; k += kHcThreads) {
    const float v = to_f(xt[k]);
    acc[HC] = fmaf(v, v, acc[HC]);
#pragma unroll
    for (int j = 0; j < HC; ++j) acc[j] = fmaf(v, fn[int64_t(j) * hcd + k], acc[j]);
  }
  block_sum(acc, red);
  if (threadIdx.x == 0) {
    const float inv_rms = rsqrtf(acc[HC] / float(hcd) + norm_eps);
#pragma unroll
    for (int c = 0; c < HC; ++c)  // (mixes * rsqrt) * scale + base, each rounded as the reference's ops are
      pre_s[c] = sigmoid_f(__fadd_rn(__fmul_rn(__fmul_rn(acc[c], inv_rms), scale[0]), base[c])) + hc_eps;
  }
  __syncthreads();
  float sq[2] = {0.f, 0.f};
  T* yt = y_out + t * dim;
  for (int j = threadIdx.x; j < dim; j += kHcThreads) {
    float y = 0.f;
#pragma unroll
    for (int c = 0; c < HC; ++c) y = __fadd_rn(y, __fmul_rn(pre_s[c], to_f(xt[c * dim + j])));  // products, then sum
    const T yt_v = from_f<T>(y);
    const float yq = to_f(yt_v);
    yt[j] = yt_v;
    ysm[j] = yq;
    sq[0] = fmaf(yq, yq, sq[0]);
    if (conf_w) sq[1] = fmaf(yq, conf_w[j], sq[1]);
  }
  block_sum(sq, red);
  if (threadIdx.x == 0 && conf_out) conf_out[t] = sq[1];
  const float r = rsqrtf(sq[0] / float(dim) + norm_eps);
  T* out = xn + t * dim;
  for (int j = threadIdx.x; j < dim; j += kHcThreads) {
    const float v = ysm[j] * r;
    out[j] = from_f<T>(weight ? weight[j] * v : v);
  }
}

template <typename T>
int launch_head(const void* x, int64_t n, int hc, int dim, const float* fn, const float* scale, const float* base,
                float norm_eps, float hc_eps, const float* weight, const float* conf_w, void* y, void* xn,
                float* conf, cudaStream_t s) {
  const size_t smem = size_t(dim) * sizeof(float);
  const T* xp = static_cast<const T*>(x);
#define DSM_HC_HEAD(H)                                                                                        \
  {                                                                                                           \
    auto k = hc_head_norm_kernel<T, H>;                                                                       \
    if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != \
                                cudaSuccess)                                                                  \
      return check_launch("hc_head_norm smem attribute");                                                     \
    k<<<unsigned(n), kHcThreads, smem, s>>>(xp, dim, fn, scale, base, norm_eps, hc_eps, weight, conf_w,       \
                                            static_cast<T*>(y), static_cast<T*>(xn), conf);                   \
    return check_launch("hc_head_norm");                                                                      \
  }
  switch (hc) {
    case 1: DSM_HC_HEAD(1)
    case 2: DSM_HC_HEAD(2)
    case 4: DSM_HC_HEAD(4)
    default: return fail(DSM_ERR_UNSUPPORTED, "dsm_hc_head_norm: hc_mult must be 1, 2 or 4");
  }
#undef DSM_HC_HEAD
}

template <typename T>
int launch_pre(const void* x, int64_t n, int hc, int dim, const float* fn, const float* scale, const float* base,
               int iters, float norm_eps, float hc_eps, const float* weight, void* xn, float* post, float* comb,
               cudaStream_t s) {
  const size_t smem = size_t(dim) * sizeof(float);
  const T* xp = static_cast<const T*>(x);
  T* xo = static_cast<T*>(xn);
  // a draft step's few tokens take two CTAs each (a cluster): one CTA per token would leave
  // most SMs idle, each reading the whole projection matrix from L2
  const bool pair = n <= int64_t(num_sms());
#define DSM_HC_PRE(H)                                                                                         \
  {                                                                                                           \
    auto k = pair ? hc_pre_norm_pair_kernel<T, H> : hc_pre_norm_kernel<T, H>;                               \
    if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != \
                                cudaSuccess)                                                                  \
      return check_launch("hc_pre_norm smem attribute");                                                      \
    k<<<unsigned(pair ? 2 * n : n), kHcThreads, smem, s>>>(xp, dim, fn, scale, base, iters, norm_eps, hc_eps,  \
                                                           weight, xo, post, comb);                           \
    return check_launch("hc_pre_norm");                                                                       \
  }
  switch (hc) {
    case 1: DSM_HC_PRE(1)
    case 2: DSM_HC_PRE(2)
    case 4: DSM_HC_PRE(4)
    default: return fail(DSM_ERR_UNSUPPORTED, "dsm_hc_pre_norm: hc_mult must be 1, 2 or 4");
  }
#undef DSM_HC_PRE
}

template <typename T>
int launch_post(const void* h, const void* res, int64_t n, int hc, int dim, const float* post, const float* comb,
                void* out, cudaStream_t s) {
  const dim3 grid(unsigned(ceil_div(dim, kHcThreads)), unsigned(n));
  const T* hp = static_cast<const T*>(h);
  const T* rp = static_cast<const T*>(res);
  T* op = static_cast<T*>(out);
  switch (hc) {
    case 1: hc_post_kernel<T, 1><<<grid, kHcThreads, 0, s>>>(hp, rp, dim, post, comb, op); break;
    case 2: hc_post_kernel<T, 2><<<grid, kHcThreads, 0, s>>>(hp, rp, dim, post, comb, op); break;
    case 4: hc_post_kernel<T, 4><<<grid, kHcThreads, 0, s>>>(hp, rp, dim, post, comb, op); break;
    default: return fail(DSM_ERR_UNSUPPORTED, "dsm_hc_post: hc_mult must be 1, 2 or 4");
  }
  return check_launch("hc_post");
}

}  // namespace
}  // namespace dsm

extern "C" int dsm_hc_pre_norm(const void* x, int x_dtype, int64_t n_tokens, int hc_mult, int dim, const float* hc_fn,
                               const float* hc_scale, const float* hc_base, int sinkhorn_iters, float norm_eps,
                               float hc_eps, const float* norm_weight, void* x_norm_out, float* post_out,
                               float* comb_out, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(n_tokens >= 0 && dim > 0 && hc_mult > 0 && sinkhorn_iters >= 1, "dsm_hc_pre_norm: bad shape");
  DSM_REQUIRE(dim <= 48 * 1024, "dsm_hc_pre_norm: dim too large for the shared-memory row");
  DSM_REQUIRE(x_dtype == DSM_DT_F32 || x_dtype == DSM_DT_BF16, "dsm_hc_pre_norm: x must be F32 or BF16");
  if (n_tokens == 0) return DSM_OK;
  DSM_REQUIRE(x && hc_fn && hc_scale && hc_base && x_norm_out && post_out && comb_out, "dsm_hc_pre_norm: NULL pointer");
  cudaStream_t s = as_stream(stream);
  if (x_dtype == DSM_DT_BF16)
    return launch_pre<__nv_bfloat16>(x, n_tokens, hc_mult, dim, hc_fn, hc_scale, hc_base, sinkhorn_iters, norm_eps,
                                     hc_eps, norm_weight, x_norm_out, post_out, comb_out, s);
  return launch_pre<float>(x, n_tokens, hc_mult, dim, hc_fn, hc_scale, hc_base, sinkhorn_iters, norm_eps, hc_eps,
                           norm_weight, x_norm_out, post_out, comb_out, s);
}

extern "C" int dsm_hc_post(const void* h, const void* residual, int dtype, int64_t n_tokens, int hc_mult, int dim,
                           const float* post, const float* comb, void* out, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(n_tokens >= 0 && dim > 0 && hc_mult > 0, "dsm_hc_post: bad shape");
  DSM_REQUIRE(dtype == DSM_DT_F32 || dtype == DSM_DT_BF16, "dsm_hc_post: dtype must be F32 or BF16");
  if (n_tokens == 0) return DSM_OK;
  DSM_REQUIRE(h && residual && post && comb && out, "dsm_hc_post: NULL pointer");
  cudaStream_t s = as_stream(stream);
  if (dtype == DSM_DT_BF16)
    return launch_post<__nv_bfloat16>(h, residual, n_tokens, hc_mult, dim, post, comb, out, s);
  return launch_post<float>(h, residual, n_tokens, hc_mult, dim, post, comb, out, s);
}

extern "C" int dsm_hc_head_norm(const void* x, int x_dtype, int64_t n_tokens, int hc_mult, int dim, const float* hc_fn,
                                const float* hc_scale, const float* hc_base, float norm_eps, float hc_eps,
                                const float* norm_weight, const float* conf_w, void* y_out, void* x_norm_out,
                                float* conf_out, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(n_tokens >= 0 && dim > 0 && hc_mult > 0, "dsm_hc_head_norm: bad shape");
  DSM_REQUIRE(dim <= 48 * 1024, "dsm_hc_head_norm: dim too large for the shared-memory row");
  DSM_REQUIRE(x_dtype == DSM_DT_F32 || x_dtype == DSM_DT_BF16, "dsm_hc_head_norm: x must be F32 or BF16");
  if (n_tokens == 0) return DSM_OK;
  DSM_REQUIRE(x && hc_fn && hc_scale && hc_base && y_out && x_norm_out, "dsm_hc_head_norm: NULL pointer");
  DSM_REQUIRE(!conf_w || conf_out, "dsm_hc_head_norm: conf_w without conf_out");
  cudaStream_t s = as_stream(stream);
  if (x_dtype == DSM_DT_BF16)
    return launch_head<__nv_bfloat16>(x, n_tokens, hc_mult, dim, hc_fn, hc_scale, hc_base, norm_eps, hc_eps,
                                      norm_weight, conf_w, y_out, x_norm_out, conf_out, s);
  return launch_head<float>(x, n_tokens, hc_mult, dim, hc_fn, hc_scale, hc_base, norm_eps, hc_eps, norm_weight, conf_w,
                            y_out, x_norm_out, conf_out, s);
}
