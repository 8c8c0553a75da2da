// The Qwen3 DSpark draft attention (dspark_mlx/arch/qwen3.py:84-143): grouped-query attention
// of the draft block over [context || block], around the packed-weight projections
// (dsm_linear):
//
//   dsm_qkv_norm_rope  a fused projection's fp32 rows [n, (n_q + 2 n_kv) * head_dim] (plus the
//                      lo rows of an fp32 input staged hi + lo): every head rounded to the
//                      activation dtype; the q and k heads RMSNormed with their weights
//                      (norm_rope.py:22-39) and rotated by NeoX half-split RoPE with the
//                      tables cast to the activation dtype (qwen3.py:64-73); q heads written
//                      [n, n_q, head_dim], k and v heads into [batch, n_kv, cap, head_dim]
//                      caches at rows row0 + t (qwen3.py:97-108, 122-137).
//   dsm_gqa_attn       softmax(q k^T * scale) v of every query head over its KV head's
//                      context rows and then the block's own rows, with no mask
//                      (mx.fast.scaled_dot_product_attention, qwen3.py:114-116, 141-143),
//                      written [batch, block, n_heads * head_dim] for o_proj.
//
// The attention is split over keys. A CTA holds one KV head's query rows (the group's heads
// x the block's tokens, up to 32) and one key range; it streams 64-key tiles of K and V
// through shared memory with an online softmax and leaves fp32 partials (m, l, acc) per row
// and range. A second kernel combines the ranges in order. The output is rounded once to the
// activation dtype. Two CTA kernels:
//   gqa_attn_kernel  fp32 CUDA-core products, any dtype and head_dim 32..256;
//   gqa_mma_kernel   bf16 with head_dim 64 or 128: K/V tiles double-buffered by cp.async,
//                    q.k and p.v on mma.m16n8k16 (bf16 in, fp32 accumulate; p rounded to
//                    bf16 for the second product), each warp an online softmax over half of
//                    every tile, so each key range leaves two partials.
// dsm_set_attn_kernel picks between them (per host thread).
#include <atomic>

#include "common.cuh"
#include "warp_mma.cuh"

namespace dsm {
namespace {

constexpr int kGqaThreads = 256;
constexpr int kGqaWarps = kGqaThreads / 32;
constexpr int kKeyTile = 64;    // keys per shared-memory tile
constexpr int kRowBlock = 32;   // query rows per CTA
constexpr int kMaxSplits = 64;  // key ranges per KV head
constexpr int kMaxParts = 2 * kMaxSplits;  // partials per query row (two per range on the mma path)
constexpr int kMaxHeadDim = 256;
constexpr int kMmaThreads = 128;  // 4 warps: 2 row tiles of 16 x 2 key halves of 32
// K/V tile slots: one load ahead of the tile being multiplied. At head_dim 128 a CTA holds
// (32 + 2 x 2 x 64) rows of 256 B = 73,728 B of shared memory, so three CTAs share an SM
// (12 warps: the warps' dependency chains, not the loads, bound this kernel).
constexpr int kMmaStages = 2;
constexpr int kMmaCtasPerSm = 3;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per (row, head). Heads [0, n_q) are queries, [n_q, n_q + n_kv) keys, then values.
// Row r belongs to sequence r / period at token t = r % period: RoPE table row tab0 + t,
// cache row row0 + t.
template <typename T>
__global__ void __launch_bounds__(kGqaThreads) qkv_norm_rope_kernel(
    const float* __restrict__ in, const float* __restrict__ in_lo, int64_t n_rows, int n_q, int n_kv, int head_dim,
    const float* __restrict__ q_w, const float* __restrict__ k_w, float eps, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, int tab0, int period, T* __restrict__ q_out, T* __restrict__ k_out,
    T* __restrict__ v_out, int kv_cap, int row0) {
  __shared__ float buf[kGqaWarps][kMaxHeadDim];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = n_q + 2 * n_kv;
  const int64_t wid = int64_t(blockIdx.x) * kGqaWarps + warp;
  if (wid >= n_rows * heads) return;  // whole warps leave; only warp-level syncs follow
  const int64_t r = wid / heads;
  const int hh = int(wid % heads);
  const int64_t off = (r * heads + hh) * int64_t(head_dim);
  float* x = buf[warp];
  float sq = 0.f;
  for (int d = lane; d < head_dim; d += 32) {
    float v = in[off + d];
    if (in_lo) v += in_lo[off + d];
    v = rnd<T>(v);  // the projection's output dtype
    x[d] = v;
    sq = fmaf(v, v, sq);
  }
  const int t = int(r % period);
  const int64_t b = r / period;
  if (hh >= n_q + n_kv) {  // a value head: the projection as it is
    const int g = hh - n_q - n_kv;
    T* dst = v_out + ((b * n_kv + g) * kv_cap + row0 + t) * int64_t(head_dim);
    for (int d = lane; d < head_dim; d += 32) dst[d] = st_f<T>(x[d]);
    return;
  }
  const float rs = rsqrtf(warp_sum(sq) / float(head_dim) + eps);
  const float* w = hh < n_q ? q_w : k_w;
  for (int d = lane; d < head_dim; d += 32) x[d] = rnd<T>(__fmul_rn(w[d], __fmul_rn(x[d], rs)));
  __syncwarp();
  const int half = head_dim / 2;
  const int64_t p = int64_t(tab0) + t;
  T* dst = hh < n_q ? q_out + (r * n_q + hh) * int64_t(head_dim)
                    : k_out + ((b * n_kv + (hh - n_q)) * kv_cap + row0 + t) * int64_t(head_dim);
  for (int d = lane; d < head_dim; d += 32) {
    // x * cos + rotate_half(x) * sin, each product and the sum rounded to T
    const float c = rnd<T>(cos_t[p * head_dim + d]);
    const float s = rnd<T>(sin_t[p * head_dim + d]);
    const float rot = d < half ? -x[d + half] : x[d - half];
    dst[d] = st_f<T>(__fadd_rn(rnd<T>(__fmul_rn(x[d], c)), rnd<T>(__fmul_rn(rot, s))));
  }
}

// Grid (split, kv head, batch * row_blocks). Local row r is query row ri = row_block * 32 + r
// of KV head g: head g * G + ri / block, token ri % block. Keys [split * chunk, +chunk) of
// the n_ctx context rows followed by the block rows.
template <typename T, int HD>
__global__ void __launch_bounds__(kGqaThreads) gqa_attn_kernel(
    const T* __restrict__ q, const T* __restrict__ ctx_k, const T* __restrict__ ctx_v, int64_t ctx_sb,
    int64_t ctx_sh, int n_ctx, const T* __restrict__ blk_k, const T* __restrict__ blk_v, int block, int n_heads,
    int n_kv, int row_blocks, int chunk, int n_splits, float scale, float* __restrict__ part,
    float* __restrict__ ml) {
  constexpr int KP = HD + 1;                           // padded K rows: conflict-free reads by key
  constexpr int RS = kGqaThreads / kKeyTile;           // row stride of the score threads
  constexpr int SR = kRowBlock / RS;                   // scores per thread per tile
  constexpr int RPP = kGqaThreads / HD;                // row stride of the P.V threads
  constexpr int NACC = kRowBlock / RPP;                // accumulators per thread
  static_assert(HD >= 32 && HD <= kMaxHeadDim && kGqaThreads % HD == 0, "head_dim");
  extern __shared__ float smem[];
  float* Qs = smem;                          // [kRowBlock][HD]
  float* Ks = Qs + kRowBlock * HD;           // [kKeyTile][KP]
  float* Vs = Ks + kKeyTile * KP;            // [kKeyTile][HD]
  float* P = Vs + kKeyTile * HD;             // [kRowBlock][kKeyTile]
  float* m_run = P + kRowBlock * kKeyTile;   // [kRowBlock]
  float* l_run = m_run + kRowBlock;          // [kRowBlock]
  float* alpha = l_run + kRowBlock;          // [kRowBlock]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, g = blockIdx.y;
  const int b = int(blockIdx.z) / row_blocks, r0 = (int(blockIdx.z) % row_blocks) * kRowBlock;
  const int G = n_heads / n_kv;
  const int nrows = min(kRowBlock, G * block - r0);
  const int nk = n_ctx + block;
  const int k0 = split * chunk, k1 = min(nk, k0 + chunk);

  for (int i = tid; i < kRowBlock * HD; i += kGqaThreads) {
    const int r = i / HD, d = i % HD;
    float v = 0.f;
    if (r < nrows) {
      const int ri = r0 + r;
      const int h = g * G + ri / block, t = ri % block;
      v = ld_f(q, ((int64_t(b) * block + t) * n_heads + h) * HD + d);
    }
    Qs[i] = v;
  }
  for (int i = tid; i < kRowBlock * kKeyTile; i += kGqaThreads) P[i] = 0.f;
  if (tid < kRowBlock) {
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.f;
    alpha[tid] = 0.f;
  }
  float acc[NACC];
#pragma unroll
  for (int i = 0; i < NACC; ++i) acc[i] = 0.f;
  const int pd = tid % HD, prow = tid / HD;              // P.V: column pd of rows prow + i * RPP
  const int sj = tid % kKeyTile, srow = tid / kKeyTile;  // scores: key sj of rows srow + i * RS
  const int64_t ctx_base = int64_t(b) * ctx_sb + int64_t(g) * ctx_sh;
  const int64_t blk_base = (int64_t(b) * n_kv + g) * block;

  for (int kt0 = k0; kt0 < k1; kt0 += kKeyTile) {
    const int kt = min(kKeyTile, k1 - kt0);
    __syncthreads();  // the previous tile is consumed (and the initial fills are visible)
    for (int i = tid; i < kKeyTile * HD; i += kGqaThreads) {
      const int j = i / HD, d = i % HD;
      float kv = 0.f, vv = 0.f;
      if (j < kt) {
        const int k = kt0 + j;
        if (k < n_ctx) {
          const int64_t o = ctx_base + int64_t(k) * HD + d;
          kv = ld_f(ctx_k, o);
          vv = ld_f(ctx_v, o);
        } else {
          const int64_t o = (blk_base + (k - n_ctx)) * HD + d;
          kv = ld_f(blk_k, o);
          vv = ld_f(blk_v, o);
        }
      }
      Ks[j * KP + d] = kv;
      Vs[j * HD + d] = vv;
    }
    __syncthreads();
    {
      float s[SR];
#pragma unroll
      for (int i = 0; i < SR; ++i) s[i] = 0.f;
      const float* kr = Ks + sj * KP;
      for (int d = 0; d < HD; ++d) {
        const float kd = kr[d];
#pragma unroll
        for (int i = 0; i < SR; ++i) s[i] = fmaf(Qs[(srow + i * RS) * HD + d], kd, s[i]);
      }
#pragma unroll
      for (int i = 0; i < SR; ++i) P[(srow + i * RS) * kKeyTile + sj] = s[i] * scale;
    }
    __syncthreads();
    for (int r = warp; r < nrows; r += kGqaWarps) {  // online softmax of row r over this tile
      float* pr = P + r * kKeyTile;
      float mt = -INFINITY;
      for (int j = lane; j < kt; j += 32) mt = fmaxf(mt, pr[j]);
      const float m_old = m_run[r];
      const float m_new = fmaxf(m_old, warp_max(mt));
      float ls = 0.f;
      for (int j = lane; j < kKeyTile; j += 32) {
        const float e = j < kt ? expf(pr[j] - m_new) : 0.f;
        pr[j] = e;
        ls += e;
      }
      ls = warp_sum(ls);
      if (lane == 0) {
        const float a = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        alpha[r] = a;
        l_run[r] = l_run[r] * a + ls;
        m_run[r] = m_new;
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NACC; ++i) acc[i] *= alpha[prow + i * RPP];
    for (int j = 0; j < kt; ++j) {
      const float v = Vs[j * HD + pd];
#pragma unroll
      for (int i = 0; i < NACC; ++i) acc[i] = fmaf(P[(prow + i * RPP) * kKeyTile + j], v, acc[i]);
    }
  }
  // partials of query row (b, h, t): part[row][split][HD], ml[row][split][2]
#pragma unroll
  for (int i = 0; i < NACC; ++i) {
    const int r = prow + i * RPP;
    if (r < nrows) {
      const int ri = r0 + r;
      const int64_t row = (int64_t(b) * n_heads + g * G + ri / block) * block + ri % block;
      part[(row * n_splits + split) * HD + pd] = acc[i];
    }
  }
  if (tid < nrows) {
    const int ri = r0 + tid;
    const int64_t row = (int64_t(b) * n_heads + g * G + ri / block) * block + ri % block;
    ml[(row * n_splits + split) * 2] = m_run[tid];
    ml[(row * n_splits + split) * 2 + 1] = l_run[tid];
  }
}

// Grid and rows as gqa_attn_kernel; bf16 only. Warp w takes row tile w & 1 (rows 16 (w & 1)
// ..) and key half w >> 1 (keys 32 (w >> 1) .. of every 64-key tile), keeps its own running
// max / denominator / output, and leaves partial 2 * split + (w >> 1). Fragment layouts are
// those of mma.m16n8k16: thread (g, t) = (lane / 4, lane % 4) holds rows g and g + 8,
// columns 2t and 2t + 1 of each 8-wide accumulator tile. Shared rows are unpadded, with the
// 16-byte chunks of row r XOR-swizzled by r % 8, so the eight rows that one 8x8 ldmatrix
// reads at a logical chunk sit in eight different bank groups. Without padding, and with
// the q fragments loaded per tile instead of held in registers, three CTAs share an SM.
template <int HD>
__global__ void __launch_bounds__(kMmaThreads, kMmaCtasPerSm) gqa_mma_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ ctx_k,
    const __nv_bfloat16* __restrict__ ctx_v, int64_t ctx_sb, int64_t ctx_sh, int n_ctx,
    const __nv_bfloat16* __restrict__ blk_k, const __nv_bfloat16* __restrict__ blk_v, int block, int n_heads,
    int n_kv, int row_blocks, int chunk, int n_parts, float scale, float* __restrict__ part,
    float* __restrict__ ml) {
  constexpr int ROWB = HD * 2;  // shared row (bytes)
  constexpr int CPR = HD / 8;    // 16-byte chunks per row
  constexpr int KS = HD / 16;  // k-steps of q.k
  constexpr int NT = HD / 8;   // 8-wide output tiles
  static_assert(HD == 64 || HD == 128, "head_dim");
  extern __shared__ __align__(128) unsigned char gqa_smem[];
  // byte offsets: q [32 rows], K [stage][64 rows], V [stage][64 rows]
  constexpr uint32_t kQ0 = 0, kK0 = kRowBlock * ROWB, kV0 = kK0 + kMmaStages * kKeyTile * ROWB;
  const uint32_t sm0 = smem_u32(gqa_smem);
  // chunk c of row r of a region at byte offset base
  auto swz = [](uint32_t base, int r, int c) -> uint32_t {
    return base + uint32_t(r * ROWB) + (uint32_t(c ^ (r & 7)) << 4);
  };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int mt = warp & 1, kh = warp >> 1;
  const int split = blockIdx.x, g = blockIdx.y;
  const int b = int(blockIdx.z) / row_blocks, r0 = (int(blockIdx.z) % row_blocks) * kRowBlock;
  const int G = n_heads / n_kv;
  const int nrows = min(kRowBlock, G * block - r0);
  const int nk = n_ctx + block;
  const int k0 = split * chunk, k1 = min(nk, k0 + chunk);
  const int n_tiles = (k1 - k0 + kKeyTile - 1) / kKeyTile;
  const int64_t ctx_base = int64_t(b) * ctx_sb + int64_t(g) * ctx_sh;
  const int64_t blk_base = (int64_t(b) * n_kv + g) * block;

  for (int i = tid; i < kRowBlock * CPR; i += kMmaThreads) {
    const int r = i / CPR, c = i % CPR;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < nrows) {
      const int ri = r0 + r;
      const int h = g * G + ri / block, t = ri % block;
      v = *reinterpret_cast<const uint4*>(q + ((int64_t(b) * block + t) * n_heads + h) * HD + c * 8);
    }
    *reinterpret_cast<uint4*>(gqa_smem + swz(kQ0, r, c)) = v;
  }
  auto load_tile = [&](int tile, int stage) {
    const int kt0 = k0 + tile * kKeyTile;
    const uint32_t ks = kK0 + uint32_t(stage * kKeyTile * ROWB), vs = kV0 + uint32_t(stage * kKeyTile * ROWB);
    if (kt0 + kKeyTile <= min(k1, n_ctx)) {
      // a whole tile of context rows (every tile but a range's last): fixed column chunk per
      // thread, rows RPP apart, no per-chunk bounds or source choice
      constexpr int RPP = kMmaThreads / CPR;
      const int c = tid % CPR, jr = tid / CPR;
      const int64_t src0 = ctx_base + int64_t(kt0 + jr) * HD + c * 8;
      // RPP is a multiple of 8: the thread's rows share one swizzle
      const uint32_t kd = sm0 + swz(ks, jr, c), vd = sm0 + swz(vs, jr, c);
#pragma unroll
      for (int it = 0; it < kKeyTile / RPP; ++it) {
        cp_async16(kd + uint32_t(it * RPP * ROWB), ctx_k + src0 + int64_t(it) * RPP * HD, true);
        cp_async16(vd + uint32_t(it * RPP * ROWB), ctx_v + src0 + int64_t(it) * RPP * HD, true);
      }
      return;
    }
    for (int i = tid; i < kKeyTile * CPR; i += kMmaThreads) {
      const int j = i / CPR, c = i % CPR;
      const int k = kt0 + j;
      const bool valid = k < k1;
      const __nv_bfloat16* ksrc;
      const __nv_bfloat16* vsrc;
      if (valid && k < n_ctx) {
        ksrc = ctx_k + ctx_base + int64_t(k) * HD + c * 8;
        vsrc = ctx_v + ctx_base + int64_t(k) * HD + c * 8;
      } else {
        const int kb = valid ? k - n_ctx : 0;  // nothing is read past the range: any in-range row
        ksrc = blk_k + (blk_base + kb) * HD + c * 8;
        vsrc = blk_v + (blk_base + kb) * HD + c * 8;
      }
      cp_async16(sm0 + swz(ks, j, c), ksrc, valid);
      cp_async16(sm0 + swz(vs, j, c), vsrc, valid);
    }
  };
  // tiles 0 .. kMmaStages - 2 ahead; one commit group per tile slot, empty or not, so the
  // wait count below holds (every range holds at least one key)
#pragma unroll
  for (int t = 0; t < kMmaStages - 1; ++t) {
    if (t < n_tiles) load_tile(t, t);
    cp_async_commit();
  }
  const int q_row = 16 * mt + (lane & 7) + 8 * ((lane >> 3) & 1);  // this lane's ldmatrix row of q

  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // m_run in base-2 units
  const float scale2 = scale * 1.4426950408889634f;  // log2(e)
  for (int tile = 0; tile < n_tiles; ++tile) {
    const int stage = tile % kMmaStages;
    // the slot refilled here held tile - 1, released by the barrier that ended its iteration
    if (tile + kMmaStages - 1 < n_tiles) load_tile(tile + kMmaStages - 1, (tile + kMmaStages - 1) % kMmaStages);
    cp_async_commit();
    cp_async_wait<kMmaStages - 1>();  // this tile's group has landed (and, at tile 0, q)
    __syncthreads();
    const int kt = min(kKeyTile, k1 - (k0 + tile * kKeyTile));
    const uint32_t ks = kK0 + uint32_t(stage * kKeyTile * ROWB), vs = kV0 + uint32_t(stage * kKeyTile * ROWB);
    const int kr0 = 32 * kh;  // this warp's key half
    float s[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t qa[4];  // q's A fragment of k-step kk
      ldsm_x4(sm0 + swz(kQ0, q_row, 2 * kk + (lane >> 4)), qa[0], qa[1], qa[2], qa[3]);
#pragma unroll
      for (int p = 0; p < 2; ++p) {  // keys 16p .. 16p + 15 of this warp's half: two 8-key tiles
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sm0 + swz(ks, kr0 + 16 * p + (lane & 7) + 8 * (lane >> 4), 2 * kk + ((lane >> 3) & 1)), b0, b1,
                b2, b3);
        mma_16816(s[2 * p], qa, b0, b1);
        mma_16816(s[2 * p + 1], qa, b2, b3);
      }
    }
    // scores in base-2 units (scale * log2 e folded in): the softmax weights are exp2 of them
    float mx[2] = {-INFINITY, -INFINITY};
    if (kt == kKeyTile) {
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          s[n][c] *= scale2;
          mx[c >> 1] = fmaxf(mx[c >> 1], s[n][c]);
        }
    } else {
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int key = 32 * kh + 8 * n + 2 * t4 + (c & 1);
          const float v = key < kt ? s[n][c] * scale2 : -INFINITY;
          s[n][c] = v;
          mx[c >> 1] = fmaxf(mx[c >> 1], v);
        }
    }
    float alpha[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      const float m_new = fmaxf(m_run[i], mx[i]);
      const float mref = m_new == -INFINITY ? 0.f : m_new;  // a row with no key yet stays empty
      alpha[i] = exp2f(m_run[i] - mref);
      m_run[i] = m_new;
      mx[i] = mref;
    }
    float ls[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        // rounded to bf16 here, so the denominator sums the weights the p.v products use
        const float pv = __bfloat162float(__float2bfloat16_rn(exp2f(s[n][c] - mx[c >> 1])));
        s[n][c] = pv;
        ls[c >> 1] += pv;
      }
    l_run[0] = l_run[0] * alpha[0] + ls[0];
    l_run[1] = l_run[1] * alpha[1] + ls[1];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {  // keys 16j .. 16j + 15: the score tiles 2j, 2j + 1 as the A operand
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * j][0], s[2 * j][1]);
      pa[1] = pack_bf16x2(s[2 * j][2], s[2 * j][3]);
      pa[2] = pack_bf16x2(s[2 * j + 1][0], s[2 * j + 1][1]);
      pa[3] = pack_bf16x2(s[2 * j + 1][2], s[2 * j + 1][3]);
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {  // output columns 16dp .. 16dp + 15
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sm0 + swz(vs, kr0 + 16 * j + (lane & 7) + 8 * ((lane >> 3) & 1), 2 * dp + (lane >> 4)), b0, b1,
                  b2, b3);
        mma_16816(o[2 * dp], pa, b0, b1);
        mma_16816(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // the next iteration refills this stage
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 1);
    l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 2);
  }
  const int pi = 2 * split + kh;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = 16 * mt + g8 + 8 * i;
    if (r < nrows) {
      const int ri = r0 + r;
      const int64_t row = (int64_t(b) * n_heads + g * G + ri / block) * block + ri % block;
      float* dst = part + (row * n_parts + pi) * HD;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        dst[8 * n + 2 * t4] = o[n][2 * i];
        dst[8 * n + 2 * t4 + 1] = o[n][2 * i + 1];
      }
      if (t4 == 0) {
        ml[(row * n_parts + pi) * 2] = m_run[i] * 0.6931471805599453f;  // back to natural units: ln(2)
        ml[(row * n_parts + pi) * 2 + 1] = l_run[i];
      }
    }
  }
}

// One warp per query row (b, h, t): the key ranges' partials combined in range order,
// divided by the total denominator, rounded to T into out[b, t, h, :].
template <typename T>
__global__ void __launch_bounds__(kGqaThreads) gqa_combine_kernel(const float* __restrict__ part,
                                                                  const float* __restrict__ ml, int64_t n_rows,
                                                                  int n_parts, int head_dim, int n_heads, int block,
                                                                  T* __restrict__ out) {
  __shared__ float wts[kGqaWarps][kMaxParts];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kGqaWarps + warp;
  if (row >= n_rows) return;  // whole warps leave; only warp-level syncs follow
  const float* mlr = ml + row * n_parts * 2;
  const float* pr = part + row * n_parts * int64_t(head_dim);
  // the first four partials of this lane's first four columns are requested before the range
  // weights are worked out: their load latency overlaps that of the (m, l) pairs
  const int d0 = 4 * lane;
  float4 v0[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    v0[i] = (d0 < head_dim && i < n_parts) ? *reinterpret_cast<const float4*>(pr + int64_t(i) * head_dim + d0)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
  float m = -INFINITY;
  for (int s = lane; s < n_parts; s += 32) m = fmaxf(m, mlr[2 * s]);
  m = warp_max(m);
  float l = 0.f;
  for (int s = lane; s < n_parts; s += 32) {
    const float w = expf(mlr[2 * s] - m);
    wts[warp][s] = w;
    l = fmaf(w, mlr[2 * s + 1], l);
  }
  l = warp_sum(l);
  __syncwarp();
  const int t = int(row % block);
  const int64_t bh = row / block;
  const int h = int(bh % n_heads);
  const int64_t b = bh / n_heads;
  T* dst = out + ((b * block + t) * n_heads + h) * int64_t(head_dim);
  // four columns per lane (head_dim is a multiple of 4, the partial rows 16-byte aligned); four
  // partials' loads in flight before their adds, which keep range order
  for (int d = d0; d < head_dim; d += 128) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    int s = 0;
    for (; s + 4 <= n_parts; s += 4) {
      float4 v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        v[i] = (d == d0 && s == 0) ? v0[i] : *reinterpret_cast<const float4*>(pr + int64_t(s + i) * head_dim + d);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float w = wts[warp][s + i];
        o.x = fmaf(v[i].x, w, o.x);
        o.y = fmaf(v[i].y, w, o.y);
        o.z = fmaf(v[i].z, w, o.z);
        o.w = fmaf(v[i].w, w, o.w);
      }
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {  // the last n_parts % 4 ranges (s + i < 4 only when s == 0)
      if (s + i >= n_parts) break;
      const float4 v =
          (d == d0 && s == 0) ? v0[i] : *reinterpret_cast<const float4*>(pr + int64_t(s + i) * head_dim + d);
      const float w = wts[warp][s + i];
      o.x = fmaf(v.x, w, o.x);
      o.y = fmaf(v.y, w, o.y);
      o.z = fmaf(v.z, w, o.z);
      o.w = fmaf(v.w, w, o.w);
    }
    dst[d] = st_f<T>(o.x / l);
    dst[d + 1] = st_f<T>(o.y / l);
    dst[d + 2] = st_f<T>(o.z / l);
    dst[d + 3] = st_f<T>(o.w / l);
  }
}

struct GqaPlan {
  int row_blocks, chunk, n_splits;
};

// Key ranges: as many as keep every CTA in one wave of per_sm CTAs per SM (the CUDA-core
// kernel fits two at head_dim 128, the tensor-core kernel three), whole tiles per range, no
// empty range. Rounding the range count up instead would leave a second, partial wave:
// 16 sequences x 8 KV heads at 3 ranges are 384 CTAs for 296 slots of two per SM.
GqaPlan gqa_plan(int batch, int block, int n_heads, int n_kv, int n_ctx, int per_sm) {
  GqaPlan p;
  p.row_blocks = int(ceil_div(int64_t(n_heads / n_kv) * block, kRowBlock));
  const int64_t nk = int64_t(n_ctx) + block;
  const int64_t base = int64_t(batch) * n_kv * p.row_blocks;
  const int64_t tiles = ceil_div(nk, kKeyTile);
  int64_t want = int64_t(per_sm) * num_sms() / base;
  want = want < 1 ? 1 : (want > kMaxSplits ? kMaxSplits : want);
  if (want > tiles) want = tiles;
  const int64_t per = ceil_div(tiles, want);
  p.chunk = int(per * kKeyTile);
  p.n_splits = int(ceil_div(nk, p.chunk));
  return p;
}

size_t gqa_smem_bytes(int hd) {
  return size_t(kRowBlock * hd + kKeyTile * (hd + 1) + kKeyTile * hd + kRowBlock * kKeyTile + 3 * kRowBlock) * 4;
}

template <typename T, int HD>
int launch_gqa(const void* q, const void* ctx_k, const void* ctx_v, int64_t sb, int64_t sh, int n_ctx,
               const void* blk_k, const void* blk_v, int batch, int block, int n_heads, int n_kv, float scale,
               const GqaPlan& p, float* part, float* ml, cudaStream_t s) {
  auto k = gqa_attn_kernel<T, HD>;
  const size_t smem = gqa_smem_bytes(HD);
  if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return check_launch("gqa_attn smem attribute");
  const dim3 grid(unsigned(p.n_splits), unsigned(n_kv), unsigned(batch * p.row_blocks));
  k<<<grid, kGqaThreads, smem, s>>>(static_cast<const T*>(q), static_cast<const T*>(ctx_k),
                                     static_cast<const T*>(ctx_v), sb, sh, n_ctx, static_cast<const T*>(blk_k),
                                     static_cast<const T*>(blk_v), block, n_heads, n_kv, p.row_blocks, p.chunk,
                                     p.n_splits, scale, part, ml);
  return check_launch("gqa_attn");
}

template <typename T>
int launch_gqa_hd(int hd, const void* q, const void* ctx_k, const void* ctx_v, int64_t sb, int64_t sh, int n_ctx,
                  const void* blk_k, const void* blk_v, int batch, int block, int n_heads, int n_kv, float scale,
                  const GqaPlan& p, float* part, float* ml, cudaStream_t s) {
  switch (hd) {
    case 32:
      return launch_gqa<T, 32>(q, ctx_k, ctx_v, sb, sh, n_ctx, blk_k, blk_v, batch, block, n_heads, n_kv, scale, p,
                               part, ml, s);
    case 64:
      return launch_gqa<T, 64>(q, ctx_k, ctx_v, sb, sh, n_ctx, blk_k, blk_v, batch, block, n_heads, n_kv, scale, p,
                               part, ml, s);
    case 128:
      return launch_gqa<T, 128>(q, ctx_k, ctx_v, sb, sh, n_ctx, blk_k, blk_v, batch, block, n_heads, n_kv, scale, p,
                                part, ml, s);
    case 256:
      return launch_gqa<T, 256>(q, ctx_k, ctx_v, sb, sh, n_ctx, blk_k, blk_v, batch, block, n_heads, n_kv, scale, p,
                                part, ml, s);
    default:
      return fail(DSM_ERR_UNSUPPORTED, "dsm_gqa_attn: head_dim must be 32, 64, 128 or 256");
  }
}

// room for two partials per range (the mma kernel's key halves), whichever kernel runs
size_t gqa_ws_bytes(int batch, int block, int n_heads, int head_dim, const GqaPlan& p) {
  const size_t rows = size_t(batch) * n_heads * block;
  return rows * size_t(2 * p.n_splits) * (size_t(head_dim) + 2) * 4;
}

size_t gqa_mma_smem_bytes(int hd) { return size_t(kRowBlock + 2 * kMmaStages * kKeyTile) * hd * 2; }

template <int HD>
int launch_gqa_mma(const void* q, const void* ctx_k, const void* ctx_v, int64_t sb, int64_t sh, int n_ctx,
                   const void* blk_k, const void* blk_v, int batch, int block, int n_heads, int n_kv, float scale,
                   const GqaPlan& p, float* part, float* ml, cudaStream_t s) {
  auto k = gqa_mma_kernel<HD>;
  const size_t smem = gqa_mma_smem_bytes(HD);
  if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return check_launch("gqa_mma smem attribute");
  const dim3 grid(unsigned(p.n_splits), unsigned(n_kv), unsigned(batch * p.row_blocks));
  using B = __nv_bfloat16;
  k<<<grid, kMmaThreads, smem, s>>>(static_cast<const B*>(q), static_cast<const B*>(ctx_k),
                                     static_cast<const B*>(ctx_v), sb, sh, n_ctx, static_cast<const B*>(blk_k),
                                     static_cast<const B*>(blk_v), block, n_heads, n_kv, p.row_blocks, p.chunk,
                                     2 * p.n_splits, scale, part, ml);
  return check_launch("gqa_mma");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace dsm

using namespace dsm;

extern "C" int dsm_qkv_norm_rope(const float* in, const float* in_lo, int64_t n_rows, int n_q, int n_kv,
                                 int head_dim, const float* q_norm_w, const float* k_norm_w, float eps,
                                 const float* cos_t, const float* sin_t, int tab_rows, int tab0, int period,
                                 void* q_out, void* k_out, void* v_out, int kv_cap, int row0, int dtype,
                                 void* stream) {
  DSM_REQUIRE(n_rows >= 0 && n_q >= 0 && n_kv > 0, "dsm_qkv_norm_rope: bad shape");
  DSM_REQUIRE(head_dim >= 2 && head_dim % 2 == 0 && head_dim <= kMaxHeadDim,
              "dsm_qkv_norm_rope: head_dim must be even and at most 256");
  DSM_REQUIRE(period > 0 && n_rows % period == 0, "dsm_qkv_norm_rope: rows must be whole sequences of period rows");
  DSM_REQUIRE(tab0 >= 0 && int64_t(tab0) + period <= tab_rows, "dsm_qkv_norm_rope: RoPE table rows out of range");
  DSM_REQUIRE(row0 >= 0 && int64_t(row0) + period <= kv_cap, "dsm_qkv_norm_rope: cache rows out of range");
  DSM_REQUIRE(dtype == DSM_DT_F32 || dtype == DSM_DT_BF16, "dsm_qkv_norm_rope: dtype must be F32 or BF16");
  if (n_rows == 0) return DSM_OK;
  DSM_REQUIRE(in && k_norm_w && cos_t && sin_t && k_out && v_out && (n_q == 0 || (q_out && q_norm_w)),
              "dsm_qkv_norm_rope: NULL pointer");
  const int64_t warps = n_rows * (n_q + 2 * int64_t(n_kv));
  const int64_t grid = ceil_div(warps, kGqaWarps);
  DSM_REQUIRE(grid <= 0x7fffffff, "dsm_qkv_norm_rope: too many rows");
  cudaStream_t s = as_stream(stream);
  if (dtype == DSM_DT_BF16)
    qkv_norm_rope_kernel<__nv_bfloat16><<<unsigned(grid), kGqaThreads, 0, s>>>(
        in, in_lo, n_rows, n_q, n_kv, head_dim, q_norm_w, k_norm_w, eps, cos_t, sin_t, tab0, period,
        static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_out), static_cast<__nv_bfloat16*>(v_out),
        kv_cap, row0);
  else
    qkv_norm_rope_kernel<float><<<unsigned(grid), kGqaThreads, 0, s>>>(
        in, in_lo, n_rows, n_q, n_kv, head_dim, q_norm_w, k_norm_w, eps, cos_t, sin_t, tab0, period,
        static_cast<float*>(q_out), static_cast<float*>(k_out), static_cast<float*>(v_out), kv_cap, row0);
  return check_launch("qkv_norm_rope");
}

extern "C" size_t dsm_gqa_attn_workspace_bytes(int batch, int block, int n_heads, int n_kv, int head_dim,
                                               int n_ctx) {
  if (batch <= 0 || block <= 0 || n_kv <= 0 || n_heads <= 0 || n_heads % n_kv != 0 || n_ctx < 0 || head_dim <= 0)
    return 0;
  // the larger of the two kernels' plans: the workspace serves either
  return gqa_ws_bytes(batch, block, n_heads, head_dim, gqa_plan(batch, block, n_heads, n_kv, n_ctx, kMmaCtasPerSm));
}

extern "C" int dsm_gqa_attn(const void* q, const void* ctx_k, const void* ctx_v, int64_t ctx_batch_stride,
                            int64_t ctx_head_stride, int n_ctx, const void* blk_k, const void* blk_v, int dtype,
                            int batch, int block, int n_heads, int n_kv, int head_dim, float scale, void* out,
                            void* ws, size_t ws_bytes, void* stream) {
  DSM_REQUIRE(batch >= 0 && block > 0 && n_kv > 0 && n_heads > 0 && n_heads % n_kv == 0,
              "dsm_gqa_attn: bad shape (n_heads must be a multiple of n_kv)");
  DSM_REQUIRE(n_ctx >= 0 && int64_t(n_ctx) + block <= 0x7fffffff, "dsm_gqa_attn: bad context length");
  DSM_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256,
              "dsm_gqa_attn: head_dim must be 32, 64, 128 or 256");
  DSM_REQUIRE(n_ctx == 0 || (ctx_batch_stride >= 0 && ctx_head_stride >= 0), "dsm_gqa_attn: bad context strides");
  DSM_REQUIRE(dtype == DSM_DT_F32 || dtype == DSM_DT_BF16, "dsm_gqa_attn: dtype must be F32 or BF16");
  if (batch == 0) return DSM_OK;
  DSM_REQUIRE(q && blk_k && blk_v && out && ws && (n_ctx == 0 || (ctx_k && ctx_v)), "dsm_gqa_attn: NULL pointer");
  DSM_REQUIRE(aligned16(ws), "dsm_gqa_attn: workspace must be 16-byte aligned");
  const int64_t rows = int64_t(batch) * n_heads * block;
  const int64_t sb = n_ctx ? ctx_batch_stride : 0, sh = n_ctx ? ctx_head_stride : 0;
  // the mma kernel moves 16-byte chunks: every row and base it reads must sit on 16 bytes
  const bool mma = attn_kernel() == 0 && dtype == DSM_DT_BF16 &&
                   (head_dim == 64 || head_dim == 128) && aligned16(q) && aligned16(blk_k) && aligned16(blk_v) &&
                   (n_ctx == 0 || (aligned16(ctx_k) && aligned16(ctx_v) && sb % 8 == 0 && sh % 8 == 0));
  const GqaPlan p = gqa_plan(batch, block, n_heads, n_kv, n_ctx, mma ? kMmaCtasPerSm : 2);
  DSM_REQUIRE(int64_t(batch) * p.row_blocks <= 65535 && n_kv <= 65535, "dsm_gqa_attn: batch or n_kv too large");
  const size_t need = gqa_ws_bytes(batch, block, n_heads, head_dim, p);
  if (ws_bytes < need) return fail(DSM_ERR_WORKSPACE, "dsm_gqa_attn: workspace too small");
  const int n_parts = mma ? 2 * p.n_splits : p.n_splits;
  float* part = static_cast<float*>(ws);
  float* ml = part + rows * n_parts * int64_t(head_dim);
  cudaStream_t s = as_stream(stream);
  int st;
  if (mma)
    st = head_dim == 64 ? launch_gqa_mma<64>(q, ctx_k, ctx_v, sb, sh, n_ctx, blk_k, blk_v, batch, block, n_heads,
                                             n_kv, scale, p, part, ml, s)
                        : launch_gqa_mma<128>(q, ctx_k, ctx_v, sb, sh, n_ctx, blk_k, blk_v, batch, block, n_heads,
                                              n_kv, scale, p, part, ml, s);
  else if (dtype == DSM_DT_BF16)
    st = launch_gqa_hd<__nv_bfloat16>(head_dim, q, ctx_k, ctx_v, sb, sh, n_ctx, blk_k, blk_v, batch, block, n_heads,
                                      n_kv, scale, p, part, ml, s);
  else
    st = launch_gqa_hd<float>(head_dim, q, ctx_k, ctx_v, sb, sh, n_ctx, blk_k, blk_v, batch, block, n_heads, n_kv,
                              scale, p, part, ml, s);
  if (st != DSM_OK) return st;
  const int64_t grid = ceil_div(rows, kGqaWarps);
  DSM_REQUIRE(grid <= 0x7fffffff, "dsm_gqa_attn: too many rows");
  if (dtype == DSM_DT_BF16)
    gqa_combine_kernel<__nv_bfloat16><<<unsigned(grid), kGqaThreads, 0, s>>>(
        part, ml, rows, n_parts, head_dim, n_heads, block, static_cast<__nv_bfloat16*>(out));
  else
    gqa_combine_kernel<float><<<unsigned(grid), kGqaThreads, 0, s>>>(part, ml, rows, n_parts, head_dim, n_heads,
                                                                     block, static_cast<float*>(out));
  return check_launch("gqa_combine");
}

namespace dsm {
namespace {
// 0 (default): the tensor-core attention kernels wherever they apply, 1: the CUDA-core kernels; per
// host thread, so one caller's choice never changes another thread's launches
thread_local int g_attn_kernel = 0;
}  // namespace
int attn_kernel() { return g_attn_kernel; }
}  // namespace dsm

extern "C" int dsm_set_attn_kernel(int kernel) {
  DSM_REQUIRE(kernel == 0 || kernel == 1, "dsm_set_attn_kernel: kernel must be 0 or 1");
  dsm::g_attn_kernel = kernel;
  return DSM_OK;
}
