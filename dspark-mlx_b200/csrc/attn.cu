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
//                       projection (attention.py:124-128).
//
// Everything is fp32 inside; values are rounded to the activation dtype where the reference's
// arrays carry it. One CTA per row (norms), per (token, head) warp (attention).
//
// sparse_attn_mma_kernel is the tensor-core form of dsm_sparse_attn for bf16 (opt-in through
// dsm_set_attn_kernel): the 64 heads of a token share one KV row set, so a CTA takes 16
// (token, head) rows of one sequence against all of its keys, streamed through shared memory
// in 32-key chunks, with q.k and p.v on mma.m16n8k16.
#include "common.cuh"
#include "warp_mma.cuh"

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
  for (int k = lane; k < nk; k += 32) {  // each weight once: the lane owning k replaces its score
    const float e = expf(sc[k] - mx);
    sc[k] = e;
    den += e;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  den += expf(sink[h] - mx);
  __syncwarp();  // every lane reads every weight below
  const int hpg = n_heads / n_groups, g = h / hpg;
  const int64_t dg = int64_t(hpg) * head_dim;
  T* oh = out + (int64_t(g) * n_tok + t) * dg + int64_t(h % hpg) * head_dim;
  const int half = rope_dim / 2, base = head_dim - rope_dim;
  for (int d0 = lane * 2; d0 < head_dim; d0 += 64) {
    float a = 0.f, c = 0.f;
    for (int k = 0; k < nk; ++k) {
      const float w = sc[k];
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

constexpr int kSaThreads = 128;   // 4 warps
constexpr int kSaChunk = 32;      // keys per shared-memory chunk
constexpr int kSaMaxKeys = 256;   // window slots + block rows
constexpr int kSaRows = 16;       // (token, head) rows per CTA

// Grid (row tile, sequence). Row r of a sequence is (token r / n_heads, head r % n_heads), so
// a tile is 16 consecutive rows of q. Keys: the window's first n_win slots, then the block's
// rows (the same rows serve as values).
// Phase 1: warp w scores keys 8w .. 8w + 7 of every chunk (q.k on mma, fp32).
// Phase 2: the row max and the softmax denominator (plus exp(sink - max)) across the four
//          warps through shared memory; p = exp(s - max) goes to shared memory as bf16.
// Phase 3: warp w takes output columns [HD/4 w, HD/4 (w + 1)) of p.v over all chunks.
// Epilogue: divide, round to bf16, inverse RoPE of the last rope_dim columns, group-major
// store as sparse_attn_kernel.
template <int HD>
__global__ void __launch_bounds__(kSaThreads) sparse_attn_mma_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ win, const __nv_bfloat16* __restrict__ blk,
    const float* __restrict__ sink, int batch, int block, int n_heads, int window, int n_win, float scale,
    int rope_dim, const float* __restrict__ cos_t, const float* __restrict__ sin_t, int pos0, int n_groups,
    __nv_bfloat16* __restrict__ out) {
  using B = __nv_bfloat16;
  constexpr int RS = HD + 8;               // shared row stride of q and key rows (elements)
  constexpr int CPR = HD / 8;              // 16-byte chunks per row
  constexpr int KS = HD / 16;              // k-steps of q.k
  constexpr int NKP = kSaMaxKeys + 8;      // shared row stride of p
  constexpr int WC = HD / 4;               // output columns per warp
  constexpr int WNT = WC / 8;              // 8-wide output tiles per warp
  constexpr int MAXC = kSaMaxKeys / kSaChunk;
  static_assert(HD % 64 == 0 && HD <= 512, "head_dim");
  extern __shared__ __align__(16) unsigned char sa_smem[];
  B* Qs = reinterpret_cast<B*>(sa_smem);            // [16][RS]
  B* Cs = Qs + kSaRows * RS;                        // [2][32][RS]
  B* Ps = Cs + 2 * kSaChunk * RS;                   // [16][NKP]
  float* red_max = reinterpret_cast<float*>(Ps + kSaRows * NKP);  // [4][16]
  float* red_sum = red_max + 4 * kSaRows;                         // [4][16]
  float* row_max = red_sum + 4 * kSaRows;                         // [16]
  float* row_den = row_max + kSaRows;                             // [16]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
  const int b = blockIdx.y;
  const int rows = block * n_heads;
  const int r0 = blockIdx.x * kSaRows;
  const int nk = n_win + block;
  const int nchunks = (nk + kSaChunk - 1) / kSaChunk;
  const int64_t qrow0 = int64_t(b) * rows + r0;

  for (int i = tid; i < kSaRows * CPR; i += kSaThreads) {
    const int r = i / CPR, c = i % CPR;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r0 + r < rows) v = *reinterpret_cast<const uint4*>(q + (qrow0 + r) * HD + c * 8);
    *reinterpret_cast<uint4*>(Qs + r * RS + c * 8) = v;
  }
  auto load_chunk = [&](int ch, int stage) {
    B* cs = Cs + stage * kSaChunk * RS;
    for (int i = tid; i < kSaChunk * CPR; i += kSaThreads) {
      const int j = i / CPR, c = i % CPR;
      const int k = ch * kSaChunk + j;
      const bool valid = k < nk;
      const B* src = (valid && k < n_win) ? win + (int64_t(b) * window + k) * HD + c * 8
                                          : blk + (int64_t(b) * block + (valid ? k - n_win : 0)) * HD + c * 8;
      cp_async16(smem_u32(cs + j * RS + c * 8), src, valid);
    }
  };

  // phase 1: scores of this warp's keys
  float s[MAXC][4];
#pragma unroll
  for (int c = 0; c < MAXC; ++c) s[c][0] = s[c][1] = s[c][2] = s[c][3] = 0.f;
  load_chunk(0, 0);
  cp_async_commit();
  __syncthreads();  // Qs
  const uint32_t qa_base = smem_u32(Qs + ((lane & 7) + 8 * ((lane >> 3) & 1)) * RS + 8 * (lane >> 4));
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    if (c < nchunks) {
      if (c + 1 < nchunks) load_chunk(c + 1, (c + 1) & 1);
      cp_async_commit();
      cp_async_wait1();
      __syncthreads();
      const uint32_t kb = smem_u32(Cs + ((c & 1) * kSaChunk + 8 * warp + (lane & 7)) * RS + 8 * (lane >> 3));
#pragma unroll 4
      for (int kk = 0; kk < KS; kk += 2) {  // two k-steps: one x4 load of 8 keys x 32 dims
        uint32_t a0[4], a1[4], b0, b1, b2, b3;
        ldsm_x4(qa_base + 32 * kk, a0[0], a0[1], a0[2], a0[3]);
        ldsm_x4(qa_base + 32 * (kk + 1), a1[0], a1[1], a1[2], a1[3]);
        ldsm_x4(kb + 32 * kk, b0, b1, b2, b3);
        mma_16816(s[c], a0, b0, b1);
        mma_16816(s[c], a1, b2, b3);
      }
      __syncthreads();  // the next iteration refills this stage
    }
  }
  // phase 2: softmax statistics across the warps, p to shared memory
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    if (c < nchunks) {
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int key = c * kSaChunk + 8 * warp + 2 * t4 + (cc & 1);
        const float v = key < nk ? s[c][cc] * scale : -INFINITY;
        s[c][cc] = v;
        mx[cc >> 1] = fmaxf(mx[cc >> 1], v);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
    mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
  }
  if (t4 == 0) {
    red_max[warp * kSaRows + g8] = mx[0];
    red_max[warp * kSaRows + g8 + 8] = mx[1];
  }
  __syncthreads();
  if (tid < kSaRows)
    row_max[tid] = fmaxf(fmaxf(red_max[tid], red_max[kSaRows + tid]),
                         fmaxf(red_max[2 * kSaRows + tid], red_max[3 * kSaRows + tid]));
  __syncthreads();
  const float m_row[2] = {row_max[g8], row_max[g8 + 8]};  // finite: every row has a valid key
  float ls[2] = {0.f, 0.f};
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    if (c < nchunks) {
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        // rounded to bf16 here, so the denominator sums the weights the p.v products use
        const float pv = __bfloat162float(__float2bfloat16_rn(expf(s[c][cc] - m_row[cc >> 1])));
        s[c][cc] = pv;
        ls[cc >> 1] += pv;
      }
      const int key = c * kSaChunk + 8 * warp + 2 * t4;
      *reinterpret_cast<uint32_t*>(Ps + g8 * NKP + key) = pack_bf16x2(s[c][0], s[c][1]);
      *reinterpret_cast<uint32_t*>(Ps + (g8 + 8) * NKP + key) = pack_bf16x2(s[c][2], s[c][3]);
    }
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    ls[i] += __shfl_xor_sync(0xffffffffu, ls[i], 1);
    ls[i] += __shfl_xor_sync(0xffffffffu, ls[i], 2);
  }
  if (t4 == 0) {
    red_sum[warp * kSaRows + g8] = ls[0];
    red_sum[warp * kSaRows + g8 + 8] = ls[1];
  }
  __syncthreads();
  if (tid < kSaRows) {
    const int r = r0 + tid;
    const int h = r < rows ? r % n_heads : 0;
    row_den[tid] = red_sum[tid] + red_sum[kSaRows + tid] + red_sum[2 * kSaRows + tid] + red_sum[3 * kSaRows + tid] +
                   expf(sink[h] - row_max[tid]);
  }
  // phase 3: p.v for this warp's columns
  float o[WNT][4];
#pragma unroll
  for (int n = 0; n < WNT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  load_chunk(0, 0);
  cp_async_commit();
  const uint32_t pa_base = smem_u32(Ps + ((lane & 7) + 8 * ((lane >> 3) & 1)) * NKP + 8 * (lane >> 4));
  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) load_chunk(c + 1, (c + 1) & 1);
    cp_async_commit();
    cp_async_wait1();
    __syncthreads();  // this chunk, and (first pass) p and the row statistics
    const uint32_t vb =
        smem_u32(Cs + ((c & 1) * kSaChunk + (lane & 7) + 8 * ((lane >> 3) & 1)) * RS + WC * warp + 8 * (lane >> 4));
#pragma unroll
    for (int j = 0; j < 2; ++j) {  // keys 16j .. 16j + 15 of the chunk
      uint32_t pa[4];
      ldsm_x4(pa_base + 2 * (c * kSaChunk + 16 * j), pa[0], pa[1], pa[2], pa[3]);
#pragma unroll
      for (int dp = 0; dp < WNT / 2; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + 2 * (16 * j * RS + 16 * dp), b0, b1, b2, b3);
        mma_16816(o[2 * dp], pa, b0, b1);
        mma_16816(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // the next iteration refills this stage
  }
  // epilogue
  const int hpg = n_heads / n_groups;
  const int64_t n_tok = int64_t(batch) * block;
  const int half = rope_dim / 2, base = HD - rope_dim;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int lr = g8 + 8 * i;
    const int r = r0 + lr;
    if (r >= rows) continue;
    const int m = r / n_heads, h = r % n_heads;
    const float den = row_den[lr];
    B* orow = out + (int64_t(h / hpg) * n_tok + int64_t(b) * block + m) * (int64_t(hpg) * HD) +
              int64_t(h % hpg) * HD;
#pragma unroll
    for (int n = 0; n < WNT; ++n) {
      const int col = WC * warp + 8 * n + 2 * t4;
      float a = rnd<B>(o[n][2 * i] / den), c = rnd<B>(o[n][2 * i + 1] / den);
      if (col >= base) rope_pair(a, c, cos_t, sin_t, pos0 + m, half, (col - base) >> 1, true);
      *reinterpret_cast<__nv_bfloat162*>(orow + col) = __floats2bfloat162_rn(a, c);
    }
  }
}

size_t sparse_mma_smem_bytes(int hd) {
  return size_t(kSaRows + 2 * kSaChunk) * (hd + 8) * 2 + size_t(kSaRows) * (kSaMaxKeys + 8) * 2 +
         size_t(4 * kSaRows * 2 + 2 * kSaRows) * 4;
}

template <int HD>
int launch_sparse_mma(const void* q, const void* win, const void* blk, const float* sink, int batch, int block,
                      int n_heads, int window, int n_win, float scale, int rope_dim, const float* cos_t,
                      const float* sin_t, int pos0, int n_groups, void* out, cudaStream_t s) {
  auto k = sparse_attn_mma_kernel<HD>;
  const size_t smem = sparse_mma_smem_bytes(HD);
  if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return check_launch("sparse_attn_mma smem attribute");
  const dim3 grid(unsigned(ceil_div(int64_t(block) * n_heads, kSaRows)), unsigned(batch));
  using B = __nv_bfloat16;
  k<<<grid, kSaThreads, smem, s>>>(static_cast<const B*>(q), static_cast<const B*>(win), static_cast<const B*>(blk),
                                   sink, batch, block, n_heads, window, n_win, scale, rope_dim, cos_t, sin_t, pos0,
                                   n_groups, static_cast<B*>(out));
  return check_launch("sparse_attn_mma");
}

bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

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
  cudaStream_t s = as_stream(stream);
  // the tensor-core kernel moves 16-byte rows and stores bf16 pairs
  const void* win_any = n_win ? window_kv : block_kv;  // never read when n_win == 0
  if (attn_kernel() == 0 && dtype == DSM_DT_BF16 && head_dim % 64 == 0 && head_dim <= 512 &&
      n_win + block <= kSaMaxKeys && batch <= 65535 && aligned_to(q, 16) && aligned_to(win_any, 16) &&
      aligned_to(block_kv, 16) && aligned_to(out, 4)) {
    switch (head_dim) {
      case 64:
        return launch_sparse_mma<64>(q, win_any, block_kv, sink, batch, block, n_heads, window, n_win, scale, rope_dim,
                                     cos_t, sin_t, pos0, n_groups, out, s);
      case 128:
        return launch_sparse_mma<128>(q, win_any, block_kv, sink, batch, block, n_heads, window, n_win, scale,
                                      rope_dim, cos_t, sin_t, pos0, n_groups, out, s);
      case 256:
        return launch_sparse_mma<256>(q, win_any, block_kv, sink, batch, block, n_heads, window, n_win, scale,
                                      rope_dim, cos_t, sin_t, pos0, n_groups, out, s);
      case 512:
        return launch_sparse_mma<512>(q, win_any, block_kv, sink, batch, block, n_heads, window, n_win, scale,
                                      rope_dim, cos_t, sin_t, pos0, n_groups, out, s);
      default:
        break;  // 192, 320, 384, 448: the CUDA-core kernel
    }
  }
  const int64_t warps = int64_t(batch) * block * n_heads;
  const unsigned grid = unsigned(ceil_div(warps * 32, kAttnThreads));
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
