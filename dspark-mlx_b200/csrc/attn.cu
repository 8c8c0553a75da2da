// The DSpark draft attention (dspark_mlx/model/attention.py, the compress_ratio == 0 MLA form)
// around the packed-weight projections (dsm_linear):
//
//   dsm_rows_norm_rope  a projection's fp32 rows (plus the lo rows of an fp32 input staged
//                       hi + lo) rounded to the activation dtype, RMSNorm with weight
//                       (norm_rope.py:22-39), and, optionally, interleaved-pair RoPE of the
//                       last rope_dim columns (norm_rope.py:52-77, attention.py:60-62) at
//                       position pos0 + row % period. Used for q_norm, kv_norm + rope.
//   dsm_q_head_norm_rope the query heads: rounded to the activation dtype, each head scaled by
//                       rsqrt(mean(q^2) + eps) with every elementwise op rounded to that
//                       dtype as MLX evaluates it (attention.py:110-111), then RoPE.
//   dsm_kv_window_write rows into the sliding KV ring: slot p % window for position p
//                       (DSparkKVCache.prefill / update, attention.py:27-57).
//   dsm_sparse_attn     gathered single-KV-head attention with the denominator-only sink
//                       (kernels.py:20-57) over the window's filled slots and the block's own
//                       rows (attention.py:65-69), then the inverse rotation of the output
//                       (attention.py:117); written group-major for the grouped output
//                       projection (attention.py:119-121).
//
// Everything is fp32 inside; values are rounded to the activation dtype where the reference's
// arrays carry it. One CTA per row (norms), per (token, head) warp (attention).
#include "common.cuh"

namespace dsm {
namespace {

constexpr int kAttnThreads = 256;

__device__ __forceinline__ float block_sum256(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < kAttnThreads / 32; ++w) s += red[w];
  return s;
}

// interleaved pair (j, j+1) of the rope slice at position pos: (re, im) rotated by +/- theta
__device__ __forceinline__ void rope_pair(float& re, float& im, const float* cos_t, const float* sin_t, int pos,
                                          int half, int k, bool inverse) {
  const float c = cos_t[int64_t(pos) * half + k];
  const float s = inverse ? -sin_t[int64_t(pos) * half + k] : sin_t[int64_t(pos) * half + k];
  // products then sum, each rounded, as the reference evaluates xr * c - xi * s and xr * s + xi * c
  const float r = __fsub_rn(__fmul_rn(re, c), __fmul_rn(im, s));
  const float i = __fadd_rn(__fmul_rn(re, s), __fmul_rn(im, c));
  re = r;
  im = i;
}

// One CTA per row: round the projection to T, RMSNorm with weight (fp32), round to T, RoPE the
// last rope_dim columns, round to T. smem: cols floats.
template <typename T>
__global__ void __launch_bounds__(kAttnThreads) rows_norm_rope_kernel(const float* __restrict__ in,
                                                                      const float* __restrict__ in_lo, int cols,
                                                                      const float* __restrict__ weight, float eps,
                                                                      int rope_dim, const float* __restrict__ cos_t,
                                                                      const float* __restrict__ sin_t, int pos0,
                                                                      int period, T* __restrict__ out) {
  extern __shared__ float row[];
  __shared__ float red[kAttnThreads / 32];
  const int64_t r = blockIdx.x;
  float sq = 0.f;
  for (int c = threadIdx.x; c < cols; c += kAttnThreads) {
    float v = in[r * cols + c];
    if (in_lo) v += in_lo[r * cols + c];
    v = rnd<T>(v);  // the projection's output dtype
    row[c] = v;
    sq = fmaf(v, v, sq);
  }
  const float rs = rsqrtf(block_sum256(sq, red) / float(cols) + eps);
  for (int c = threadIdx.x; c < cols; c += kAttnThreads) {
    const float v = row[c] * rs;
    row[c] = rnd<T>(weight ? weight[c] * v : v);
  }
  __syncthreads();
  const int half = rope_dim / 2, base = cols - rope_dim;
  const int pos = pos0 + int(r % period);
  for (int c = threadIdx.x; c < cols; c += kAttnThreads) {
    float v = row[c];
    if (c >= base) {
      const int k = (c - base) >> 1;
      float re = row[base + 2 * k], im = row[base + 2 * k + 1];
      rope_pair(re, im, cos_t, sin_t, pos, half, k, false);
      v = ((c - base) & 1) ? im : re;
    }
    out[r * cols + c] = st_f<T>(v);
  }
}

// One warp per (row, head): the head rounded to T, scaled by rsqrt(mean(q^2) + eps) with each
// op rounded to T, then RoPE of its last rope_dim dims. Lane-strided over head_dim.
template <typename T>
__global__ void __launch_bounds__(kAttnThreads) q_head_norm_rope_kernel(const float* __restrict__ in,
                                                                        const float* __restrict__ in_lo,
                                                                        int64_t n_rows, int n_heads, int head_dim,
                                                                        float eps, int rope_dim,
                                                                        const float* __restrict__ cos_t,
                                                                        const float* __restrict__ sin_t, int pos0,
                                                                        int period, T* __restrict__ out) {
  const int64_t wid = (int64_t(blockIdx.x) * kAttnThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= n_rows * n_heads) return;
  const int64_t r = wid / n_heads;
  const int64_t off = wid * head_dim;
  float sq = 0.f;
  for (int d = lane; d < head_dim; d += 32) {
    float v = in[off + d];
    if (in_lo) v += in_lo[off + d];
    v = rnd<T>(v);
    sq += rnd<T>(v * v);  // q * q in T, summed in fp32 (MLX's mean accumulates in fp32)
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float ms = rnd<T>(rnd<T>(sq / float(head_dim)) + eps);
  const float rs = rnd<T>(rsqrtf(ms));
  const int half = rope_dim / 2, base = head_dim - rope_dim;
  const int pos = pos0 + int(r % period);
  for (int d0 = lane * 2; d0 < head_dim; d0 += 64) {  // pairs (d0, d0 + 1): rope pairs are aligned
    float a = in[off + d0], b = in[off + d0 + 1];
    if (in_lo) {
      a += in_lo[off + d0];
      b += in_lo[off + d0 + 1];
    }
    a = rnd<T>(rnd<T>(a) * rs);
    b = rnd<T>(rnd<T>(b) * rs);
    if (d0 >= base) rope_pair(a, b, cos_t, sin_t, pos, half, (d0 - base) >> 1, false);
    out[off + d0] = st_f<T>(a);
    out[off + d0 + 1] = st_f<T>(b);
  }
}

// out = T(in + in_lo): a projection's fp32 rows in the activation dtype
template <typename T>
__global__ void round_rows_kernel(const float* __restrict__ in, const float* __restrict__ in_lo, int64_t n,
                                  T* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = st_f<T>(in_lo ? in[i] + in_lo[i] : in[i]);
}

// window[b, slot(p), :] = rows[b, j, :] for the rows j with slot (pos0 + j) % window
template <typename T>
__global__ void kv_window_write_kernel(const T* __restrict__ rows, int batch, int n, int dim, int pos0, int window,
                                       T* __restrict__ win) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= int64_t(batch) * n * dim) return;
  const int d = int(i % dim);
  const int64_t bj = i / dim;
  const int j = int(bj % n), b = int(bj / n);
  const int slot = (pos0 + j) % window;
  win[(int64_t(b) * window + slot) * dim + d] = rows[i];
}

// One warp per (token, head). Keys: the window's first n_win slots, then the block's rows.
// scores = q . k * scale (fp32), a softmax whose denominator adds exp(sink - max), the
// weighted sum of the rows, rounded to T, then the inverse RoPE of the last rope_dim dims.
// Output group-major: out[g][token][(head % hpg) * head_dim + d], hpg = n_heads / n_groups.
template <typename T>
__global__ void __launch_bounds__(kAttnThreads) sparse_attn_kernel(
    const T* __restrict__ q, const T* __restrict__ win, const T* __restrict__ blk, const float* __restrict__ sink,
    int batch, int block, int n_heads, int head_dim, int window, int n_win, float scale, int rope_dim,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int pos0, int n_groups, T* __restrict__ out,
    float* __restrict__ scratch) {
  const int64_t wid = (int64_t(blockIdx.x) * kAttnThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n_tok = int64_t(batch) * block;
  if (wid >= n_tok * n_heads) return;
  const int64_t t = wid / n_heads;
  const int h = int(wid % n_heads);
  const int b = int(t / block), m = int(t % block);
  const int nk = n_win + block;
  float* sc = scratch + wid * int64_t(nk);  // this warp's scores
  const T* qh = q + (t * n_heads + h) * int64_t(head_dim);
  auto key = [&](int k) -> const T* {
    return k < n_win ? win + (int64_t(b) * window + k) * head_dim : blk + (int64_t(b) * block + (k - n_win)) * head_dim;
  };
  float mx = -INFINITY;
  for (int k = 0; k < nk; ++k) {
    const T* kr = key(k);
    float s = 0.f;
    for (int d = lane; d < head_dim; d += 32) s = fmaf(ld_f(qh, d), ld_f(kr, d), s);
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    s *= scale;
    if (lane == 0) sc[k] = s;
    mx = fmaxf(mx, s);
  }
  __syncwarp();
  float den = 0.f;
  for (int k = lane; k < nk; k += 32) den += expf(sc[k] - mx);
#pragma unroll
  for (int o = 16; o; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  den += expf(sink[h] - mx);
  const int hpg = n_heads / n_groups, g = h / hpg;
  const int64_t dg = int64_t(hpg) * head_dim;
  T* oh = out + (int64_t(g) * n_tok + t) * dg + int64_t(h % hpg) * head_dim;
  const int half = rope_dim / 2, base = head_dim - rope_dim;
  for (int d0 = lane * 2; d0 < head_dim; d0 += 64) {
    float a = 0.f, c = 0.f;
    for (int k = 0; k < nk; ++k) {
      const float w = expf(sc[k] - mx);
      const T* kr = key(k);
      a = fmaf(w, ld_f(kr, d0), a);
      c = fmaf(w, ld_f(kr, d0 + 1), c);
    }
    a = rnd<T>(a / den);
    c = rnd<T>(c / den);
    if (d0 >= base) rope_pair(a, c, cos_t, sin_t, pos0 + m, half, (d0 - base) >> 1, true);
    oh[d0] = st_f<T>(a);
    oh[d0 + 1] = st_f<T>(c);
  }
}

}  // namespace
}  // namespace dsm

using namespace dsm;

extern "C" int dsm_rows_norm_rope(const float* in, const float* in_lo, int64_t n_rows, int cols, const float* weight,
                                  float eps, int rope_dim, const float* cos_t, const float* sin_t, int pos0, int period,
                                  void* out, int out_dtype, void* stream) {
  DSM_REQUIRE(n_rows >= 0 && cols > 0 && cols <= 48 * 1024, "dsm_rows_norm_rope: bad shape");
  DSM_REQUIRE(rope_dim >= 0 && rope_dim % 2 == 0 && rope_dim <= cols, "dsm_rows_norm_rope: bad rope_dim");
  DSM_REQUIRE(rope_dim == 0 || (cos_t && sin_t && period > 0 && pos0 >= 0), "dsm_rows_norm_rope: rope tables");
  DSM_REQUIRE(out_dtype == DSM_DT_F32 || out_dtype == DSM_DT_BF16, "dsm_rows_norm_rope: out must be F32 or BF16");
  if (n_rows == 0) return DSM_OK;
  DSM_REQUIRE(in && out, "dsm_rows_norm_rope: NULL pointer");
  const size_t smem = size_t(cols) * 4;
  cudaStream_t s = as_stream(stream);
  const int per = rope_dim ? period : 1;
  if (out_dtype == DSM_DT_BF16) {
    auto k = rows_norm_rope_kernel<__nv_bfloat16>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
      return check_launch("rows_norm_rope smem attribute");
    k<<<unsigned(n_rows), kAttnThreads, smem, s>>>(in, in_lo, cols, weight, eps, rope_dim, cos_t, sin_t, pos0, per,
                                                   static_cast<__nv_bfloat16*>(out));
  } else {
    auto k = rows_norm_rope_kernel<float>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
      return check_launch("rows_norm_rope smem attribute");
    k<<<unsigned(n_rows), kAttnThreads, smem, s>>>(in, in_lo, cols, weight, eps, rope_dim, cos_t, sin_t, pos0, per,
                                                   static_cast<float*>(out));
  }
  return check_launch("rows_norm_rope");
}

extern "C" int dsm_q_head_norm_rope(const float* in, const float* in_lo, int64_t n_rows, int n_heads, int head_dim,
                                    float eps, int rope_dim, const float* cos_t, const float* sin_t, int pos0,
                                    int period, void* out, int out_dtype, void* stream) {
  DSM_REQUIRE(n_rows >= 0 && n_heads > 0 && head_dim > 0 && head_dim % 2 == 0, "dsm_q_head_norm_rope: bad shape");
  DSM_REQUIRE(rope_dim >= 0 && rope_dim % 2 == 0 && rope_dim <= head_dim, "dsm_q_head_norm_rope: bad rope_dim");
  DSM_REQUIRE(rope_dim == 0 || (cos_t && sin_t && period > 0 && pos0 >= 0), "dsm_q_head_norm_rope: rope tables");
  DSM_REQUIRE(out_dtype == DSM_DT_F32 || out_dtype == DSM_DT_BF16, "dsm_q_head_norm_rope: out must be F32 or BF16");
  if (n_rows == 0) return DSM_OK;
  DSM_REQUIRE(in && out, "dsm_q_head_norm_rope: NULL pointer");
  const int64_t warps = n_rows * n_heads;
  const unsigned grid = unsigned(ceil_div(warps * 32, kAttnThreads));
  const int per = rope_dim ? period : 1;
  cudaStream_t s = as_stream(stream);
  if (out_dtype == DSM_DT_BF16)
    q_head_norm_rope_kernel<__nv_bfloat16><<<grid, kAttnThreads, 0, s>>>(in, in_lo, n_rows, n_heads, head_dim, eps,
                                                                        rope_dim, cos_t, sin_t, pos0, per,
                                                                        static_cast<__nv_bfloat16*>(out));
  else
    q_head_norm_rope_kernel<float><<<grid, kAttnThreads, 0, s>>>(in, in_lo, n_rows, n_heads, head_dim, eps, rope_dim,
                                                                cos_t, sin_t, pos0, per, static_cast<float*>(out));
  return check_launch("q_head_norm_rope");
}

extern "C" int dsm_kv_window_write(const void* rows, int dtype, int batch, int n, int dim, int pos0, int window,
                                   void* win, void* stream) {
  DSM_REQUIRE(batch >= 0 && n >= 0 && dim > 0 && window > 0 && pos0 >= 0 && n <= window,
              "dsm_kv_window_write: bad shape (at most window rows per call)");
  DSM_REQUIRE(dtype == DSM_DT_F32 || dtype == DSM_DT_BF16, "dsm_kv_window_write: dtype must be F32 or BF16");
  const int64_t total = int64_t(batch) * n * dim;
  if (total == 0) return DSM_OK;
  DSM_REQUIRE(rows && win, "dsm_kv_window_write: NULL pointer");
  const unsigned grid = unsigned(ceil_div(total, 256));
  cudaStream_t s = as_stream(stream);
  if (dtype == DSM_DT_BF16)
    kv_window_write_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(rows), batch, n, dim,
                                                               pos0, window, static_cast<__nv_bfloat16*>(win));
  else
    kv_window_write_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(rows), batch, n, dim, pos0, window,
                                                       static_cast<float*>(win));
  return check_launch("kv_window_write");
}

extern "C" size_t dsm_sparse_attn_scratch_bytes(int batch, int block, int n_heads, int n_win) {
  return size_t(batch) * block * n_heads * size_t(n_win + block) * 4;
}

extern "C" int dsm_sparse_attn(const void* q, const void* window_kv, const void* block_kv, int dtype, const float* sink,
                               int batch, int block, int n_heads, int head_dim, int window, int n_win, float scale,
                               int rope_dim, const float* cos_t, const float* sin_t, int pos0, int n_groups, void* out,
                               float* scratch, void* stream) {
  DSM_REQUIRE(batch >= 0 && block > 0 && n_heads > 0 && head_dim > 0 && head_dim % 2 == 0,
              "dsm_sparse_attn: bad shape");
  DSM_REQUIRE(n_win >= 0 && n_win <= window, "dsm_sparse_attn: n_win must be in [0, window]");
  DSM_REQUIRE(n_groups > 0 && n_heads % n_groups == 0, "dsm_sparse_attn: n_heads must be a multiple of n_groups");
  DSM_REQUIRE(rope_dim >= 0 && rope_dim % 2 == 0 && rope_dim <= head_dim, "dsm_sparse_attn: bad rope_dim");
  DSM_REQUIRE(rope_dim == 0 || (cos_t && sin_t && pos0 >= 0), "dsm_sparse_attn: rope tables");
  DSM_REQUIRE(dtype == DSM_DT_F32 || dtype == DSM_DT_BF16, "dsm_sparse_attn: dtype must be F32 or BF16");
  if (batch == 0) return DSM_OK;
  DSM_REQUIRE(q && block_kv && sink && out && scratch && (n_win == 0 || window_kv), "dsm_sparse_attn: NULL pointer");
  const int64_t warps = int64_t(batch) * block * n_heads;
  const unsigned grid = unsigned(ceil_div(warps * 32, kAttnThreads));
  cudaStream_t s = as_stream(stream);
  if (dtype == DSM_DT_BF16)
    sparse_attn_kernel<__nv_bfloat16><<<grid, kAttnThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(window_kv),
        static_cast<const __nv_bfloat16*>(block_kv), sink, batch, block, n_heads, head_dim, window, n_win, scale,
        rope_dim, cos_t, sin_t, pos0, n_groups, static_cast<__nv_bfloat16*>(out), scratch);
  else
    sparse_attn_kernel<float><<<grid, kAttnThreads, 0, s>>>(
        static_cast<const float*>(q), static_cast<const float*>(window_kv), static_cast<const float*>(block_kv), sink,
        batch, block, n_heads, head_dim, window, n_win, scale, rope_dim, cos_t, sin_t, pos0, n_groups,
        static_cast<float*>(out), scratch);
  return check_launch("sparse_attn");
}

extern "C" int dsm_round_rows(const float* in, const float* in_lo, int64_t n, void* out, int out_dtype, void* stream) {
  DSM_REQUIRE(n >= 0, "dsm_round_rows: bad size");
  DSM_REQUIRE(out_dtype == DSM_DT_F32 || out_dtype == DSM_DT_BF16, "dsm_round_rows: out must be F32 or BF16");
  if (n == 0) return DSM_OK;
  DSM_REQUIRE(in && out, "dsm_round_rows: NULL pointer");
  const unsigned grid = unsigned(ceil_div(n, 256));
  if (out_dtype == DSM_DT_BF16)
    round_rows_kernel<__nv_bfloat16><<<grid, 256, 0, as_stream(stream)>>>(in, in_lo, n, static_cast<__nv_bfloat16*>(out));
  else
    round_rows_kernel<float><<<grid, 256, 0, as_stream(stream)>>>(in, in_lo, n, static_cast<float*>(out));
  return check_launch("round_rows");
}
