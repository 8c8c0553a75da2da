// The DSpark draft head (dspark_mlx/model/block.py:103-116 with the drafter's LM head,
// dspark_mlx/model/drafter.py:29): hc_head + final RMSNorm (hc.cu), the LM head over the
// vocabulary (a packed-weight product, dsm_linear), then the left-to-right block walk
// (dspark_mlx/recipe.py:30-63): per draft position, the Markov transition bias
// (dspark_mlx/model/heads.py:11-31) of the previous token is added to the base logits and
// the next token is sampled. The confidence head (heads.py:34-49) scores each position.
//
// The walk is one cooperative launch, one CTA per SM, each CTA owning a slice of the
// vocabulary. For each position every CTA:
//   1. gathers the Markov embeddings w1[prev_b] of the batch (shared memory);
//   2. computes the rank-r bias w2[v] . e_b of its slice, adds the base logits, writes
//      the biased logits, and keeps the best candidate per batch row;
//   3. meets the other CTAs at a grid barrier. The barrier is bounded: a wait past ~2 s
//      sets the device error and ends the kernel. Then every CTA reads all candidates and
//      takes the same choice.
// Ties go to the lowest vocabulary index, as argmax does. Above temperature 0 the sampler
// is the reference's Gumbel-max over softmax probabilities: two more grid-wide reductions
// (maximum, then the sum of exponentials), with uniforms supplied by the caller.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>

#include "common.cuh"

namespace dsm {
namespace {

constexpr int kWalkThreads = 256;  // the Markov head kernel's block; the walk gives each CTA at least this many words
constexpr int kWalkCtaBound = 160;  // at least the SM count: sizes the candidate buffers
constexpr size_t kWalkHeader = 256;

struct WalkArgs {
  const float* logits;  // base logits [rows, vocab]; position (b, i) is row b * block + i
  int64_t lo_offset;    // > 0: plus row lo_offset + t (an fp32 input staged as hi + lo rows)
  int batch, block, vocab, rank, slice;
  const void* w1;
  const void* w2;
  int w_bf16;
  const void* anchor;
  int anchor_i64;
  float temperature;      // 0: argmax
  const float* uniforms;  // [block][batch][vocab] when temperature > 0
  const float* conf_part; // [batch * block] hidden half of the confidence, or NULL
  const float* conf_wr;   // [rank] Markov half of the confidence weights, or NULL
  float conf_bias;
  int32_t* out_ids;   // [batch, block + 1]
  float* biased;      // [batch, block, vocab]
  float* confidence;  // [batch, block] or NULL
  unsigned* bar;      // [2]: arrivals, completed generation; zero at launch
  int* abort_flag;    // zero at launch
  float* cand_v;      // [2][gridDim][batch]
  int* cand_i;
};

__device__ __forceinline__ float wload(const void* w, int bf16, int64_t i) {
  return bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(w)[i]) : static_cast<const float*>(w)[i];
}

// 8 consecutive weights (i a multiple of 8)
__device__ __forceinline__ void wload8(const void* w, int bf16, int64_t i, float (&o)[8]) {
  if (bf16) {
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(w) + i);
    const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[2 * j] = __uint_as_float(q[j] << 16);
      o[2 * j + 1] = __uint_as_float(q[j] & 0xFFFF0000u);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(w) + i);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(w) + i + 4);
    o[0] = a.x, o[1] = a.y, o[2] = a.z, o[3] = a.w, o[4] = b.x, o[5] = b.y, o[6] = b.z, o[7] = b.w;
  }
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// D += A (16x16 bf16, row) * B (16x8 bf16, col), fp32 accumulate
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Grid barrier over the cooperative launch. Generation g completes when g * gridDim.x
// arrivals are counted. Thread 0 waits with a ~2 s budget and an abort flag that any CTA
// can raise. Every thread gets the same verdict.
__device__ bool walk_sync(const WalkArgs& a, unsigned& gen) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned target = gen + 1;
    __threadfence();
    const unsigned arrived = atomicAdd(&a.bar[0], 1u) + 1u;
    if (arrived == target * gridDim.x) {
      __threadfence();
      atomicExch(&a.bar[1], target);
    } else {
      const uint64_t t0 = global_timer_ns();
      while (*reinterpret_cast<volatile unsigned*>(&a.bar[1]) < target) {
        if (*reinterpret_cast<volatile int*>(a.abort_flag)) {
          ok = 0;
          break;
        }
        if (global_timer_ns() - t0 > 2000000000ull) {
          raise_device_error(DSM_DEV_ERR_PIPELINE_TIMEOUT);
          atomicExch(a.abort_flag, 1);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
    gen = target;
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

// per-batch-row (value, index) maximum over the warp into sv/si[warp][b]
template <int MAXB>
__device__ __forceinline__ void warp_best(const float (&bv)[MAXB], const int (&bi)[MAXB], int batch,
                                          float (*sv)[MAXB], int (*si)[MAXB]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int b = 0; b < MAXB; ++b) {
    if (b >= batch) break;
    float v = bv[b];
    int ix = bi[b];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
      if (better(ov, oi, v, ix)) {
        v = ov;
        ix = oi;
      }
    }
    if (lane == 0) {
      sv[warp][b] = v;
      si[warp][b] = ix;
    }
  }
}

// the warps' candidates in sv/si combined: threads b < batch return row b's winner
template <int MAXB, int WARPS>
__device__ __forceinline__ void warps_best(int batch, float (*sv)[MAXB], int (*si)[MAXB], float& out_v, int& out_i) {
  __syncthreads();
  if (int(threadIdx.x) < batch) {
    const int b = threadIdx.x;
    float v = sv[0][b];
    int ix = si[0][b];
    for (int w = 1; w < WARPS; ++w)
      if (better(sv[w][b], si[w][b], v, ix)) {
        v = sv[w][b];
        ix = si[w][b];
      }
    out_v = v;
    out_i = ix;
  }
}

template <int MAXB, int WARPS>
__device__ __forceinline__ void block_sum_b(const float (&s)[MAXB], int batch, float (*sv)[MAXB], float& out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int b = 0; b < MAXB; ++b) {
    if (b >= batch) break;
    float v = s[b];
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sv[warp][b] = v;
  }
  __syncthreads();
  if (int(threadIdx.x) < batch) {
    float v = 0.f;
    for (int w = 0; w < WARPS; ++w) v += sv[w][threadIdx.x];
    out = v;
  }
}

// The CTAs' candidates for batch row b (generation buffer buf) combined by one warp: each
// lane reads every 32nd CTA (independent loads), then a shuffle reduction in value order,
// ties to the lowest index. Every lane returns the winner.
__device__ __forceinline__ void combine_best(const WalkArgs& a, int buf, int b, float& v, int& ix) {
  const int G = gridDim.x, B = a.batch, lane = threadIdx.x & 31;
  v = -INFINITY;
  ix = INT_MAX;
  for (int c = lane; c < G; c += 32) {
    const float ov = __ldcg(&a.cand_v[(int64_t(buf) * G + c) * B + b]);
    const int oi = __ldcg(&a.cand_i[(int64_t(buf) * G + c) * B + b]);
    if (better(ov, oi, v, ix)) {
      v = ov;
      ix = oi;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
    if (better(ov, oi, v, ix)) {
      v = ov;
      ix = oi;
    }
  }
}

// sum of the CTAs' partial sums for batch row b, in CTA order within each lane's share
// and then a fixed shuffle tree: the same on every CTA and every run
__device__ __forceinline__ float combine_sum(const WalkArgs& a, int buf, int b) {
  const int G = gridDim.x, B = a.batch, lane = threadIdx.x & 31;
  float z = 0.f;
  for (int c = lane; c < G; c += 32) z += __ldcg(&a.cand_v[(int64_t(buf) * G + c) * B + b]);
#pragma unroll
  for (int o = 16; o; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  return z;
}

__host__ __device__ __forceinline__ int walk_e_floats(int batch, int rank, int maxb) {
  const int f32 = batch * rank, bf = (maxb * (rank + 8) + 1) / 2;
  return f32 > bf ? f32 : bf;
}

template <int MAXB, int THREADS>
__global__ void __launch_bounds__(THREADS) head_walk_kernel(const WalkArgs a) {
  constexpr int kWarps = THREADS / 32;
  extern __shared__ float sm[];
  const int B = a.batch, R = a.rank, V = a.vocab, S = a.block;
  // Markov embeddings of the previous tokens: [B][R] fp32, or [MAXB][R + 8] bf16 (tensor-core
  // path); then [B][slice] biased logits of this slice (sampling only)
  float* e_sm = sm;
  float* li_sm = sm + walk_e_floats(B, R, MAXB);
  __shared__ int prev_s[MAXB];
  __shared__ float stat_m[MAXB], stat_z[MAXB];
  __shared__ float sv[kWarps][MAXB];
  __shared__ int si[kWarps][MAXB];
  const int G = gridDim.x;
  const int v0 = blockIdx.x * a.slice, v1 = min(V, v0 + a.slice);
  const bool sampled = a.temperature > 0.f;
  const float tp = fmaxf(a.temperature, 1e-5f);
  unsigned gen = 0;
  int buf = 0;
  if (int(threadIdx.x) < B) {
    const int b = threadIdx.x;
    const int64_t id = a.anchor_i64 ? static_cast<const int64_t*>(a.anchor)[b] : static_cast<const int32_t*>(a.anchor)[b];
    int p = int(id);
    if (id < 0 || id >= V) {
      raise_device_error(DSM_DEV_ERR_TOKEN_RANGE);
      p = 0;
    }
    prev_s[b] = p;
    if (blockIdx.x == 0) a.out_ids[int64_t(b) * (S + 1)] = p;
  }
  __syncthreads();

  // bf16 tables (rank a multiple of 32) take the tensor-core path: warp tiles of 16 vocabulary rows x 8 batch rows,
  // mma.m16n8k16 over the rank. Each lane loads 16 contiguous bytes of its two rows per 32
  // rank entries. The k order inside each 32-entry block is permuted identically in both
  // operands so that these bytes are the A fragments (lane q holds entries 8q .. 8q+7);
  // the sum over the rank is unchanged.
  const bool use_mma = a.w_bf16 != 0 && R % 32 == 0;  // whole 32-entry blocks of the rank
  constexpr int NT = MAXB / 8;
  const int RP = R + 8;  // padded row of the bf16 embeddings: conflict-free fragment loads
  __nv_bfloat16* eb = reinterpret_cast<__nv_bfloat16*>(e_sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int i = 0; i < S; ++i) {
    if (use_mma) {
      const __nv_bfloat16* w1b = static_cast<const __nv_bfloat16*>(a.w1);
      for (int k = threadIdx.x; k < NT * 8 * RP; k += THREADS) {
        const int b = k / RP, r = k - b * RP;
        eb[k] = (b < B && r < R) ? w1b[int64_t(prev_s[b]) * R + r] : __float2bfloat16_rn(0.f);
      }
    } else {
      for (int k = threadIdx.x; k < B * R; k += THREADS) {
        const int b = k / R;
        e_sm[k] = wload(a.w1, a.w_bf16, int64_t(prev_s[b]) * R + (k - b * R));
      }
    }
    __syncthreads();
    auto emit_l = [&](int b, int v, float li, float& bv, int& bi) {  // biased logit of (b, v): store, keep the best
      const int64_t t = int64_t(b) * S + i;
      a.biased[t * V + v] = li;
      if (sampled) {
        li_sm[b * a.slice + (v - v0)] = li;
        bv = fmaxf(bv, li / tp);
      } else if (li > bv) {
        bv = li;
        bi = v;
      }
    };
    auto emit = [&](int b, int v, float bias, float& bv, int& bi) {  // base logit of (b, v) plus the bias
      const int64_t t = int64_t(b) * S + i;
      float l = a.logits[t * V + v];
      if (a.lo_offset) l += a.logits[(a.lo_offset + t) * V + v];
      emit_l(b, v, l + bias, bv, bi);
    };
    if (use_mma) {
      const int g = lane >> 2, q = lane & 3;
      const __nv_bfloat16* w2b = static_cast<const __nv_bfloat16*>(a.w2);
      float bv2[NT][2];
      int bi2[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          bv2[nt][c] = -INFINITY;
          bi2[nt][c] = INT_MAX;
        }
      for (int tile = warp; v0 + tile * 16 < v1; tile += kWarps) {
        const int ra = v0 + tile * 16 + g, rb = ra + 8;
        const bool oka = ra < v1, okb = rb < v1;
        // The tile's base logits and its Markov rows for up to 256 rank entries are all
        // requested before the first product: one memory latency per tile, not one per
        // 128 entries plus one for the logits.
        float lg[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt * 8 >= B) break;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int b = nt * 8 + 2 * q + c;
            const int64_t t = int64_t(b) * S + i;
            lg[nt][c] = lg[nt][2 + c] = 0.f;
            if (b >= B) continue;
            if (oka) lg[nt][c] = __ldg(&a.logits[t * V + ra]) + (a.lo_offset ? __ldg(&a.logits[(a.lo_offset + t) * V + ra]) : 0.f);
            if (okb) lg[nt][2 + c] = __ldg(&a.logits[t * V + rb]) + (a.lo_offset ? __ldg(&a.logits[(a.lo_offset + t) * V + rb]) : 0.f);
          }
        }
        float d[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) d[nt][0] = d[nt][1] = d[nt][2] = d[nt][3] = 0.f;
        for (int k8 = 0; k8 < R; k8 += 256) {  // eight 32-entry blocks: their 16 loads in flight together
          const uint4 z = make_uint4(0u, 0u, 0u, 0u);
          uint4 A0[8], A1[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int k2 = k8 + 32 * u;
            A0[u] = (oka && k2 < R) ? __ldg(reinterpret_cast<const uint4*>(w2b + int64_t(ra) * R + k2 + 8 * q)) : z;
            A1[u] = (okb && k2 < R) ? __ldg(reinterpret_cast<const uint4*>(w2b + int64_t(rb) * R + k2 + 8 * q)) : z;
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int k2 = k8 + 32 * u;
            if (k2 >= R) break;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if (nt * 8 >= B) break;
              const uint4 Bv = *reinterpret_cast<const uint4*>(eb + (nt * 8 + g) * RP + k2 + 8 * q);
              mma_bf16_16816(d[nt], A0[u].x, A1[u].x, A0[u].y, A1[u].y, Bv.x, Bv.y);
              mma_bf16_16816(d[nt], A0[u].z, A1[u].z, A0[u].w, A1[u].w, Bv.z, Bv.w);
            }
          }
        }
        // D fragment: d0, d1 row ra; d2, d3 row rb; batch nt*8 + 2q + {0, 1}
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt * 8 >= B) break;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int b = nt * 8 + 2 * q + c;
            if (b >= B) continue;
            if (oka) emit_l(b, ra, lg[nt][c] + d[nt][c], bv2[nt][c], bi2[nt][c]);
            if (okb) emit_l(b, rb, lg[nt][2 + c] + d[nt][2 + c], bv2[nt][c], bi2[nt][c]);
          }
        }
      }
      // the warp's best per batch row: lanes of equal q hold the same batch columns
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (nt * 8 >= B) break;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v = bv2[nt][c];
          int ix = bi2[nt][c];
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
            if (better(ov, oi, v, ix)) {
              v = ov;
              ix = oi;
            }
          }
          const int b = nt * 8 + 2 * q + c;
          if (g == 0 && b < B) {
            sv[warp][b] = v;
            si[warp][b] = ix;
          }
        }
      }
    } else {
      float best[MAXB];
      int bidx[MAXB];
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        best[b] = -INFINITY;
        bidx[b] = INT_MAX;
      }
      for (int v = v0 + threadIdx.x; v < v1; v += THREADS) {
        float acc[MAXB];
#pragma unroll
        for (int b = 0; b < MAXB; ++b) acc[b] = 0.f;
        for (int r = 0; r < R; r += 8) {
          float w[8];
          wload8(a.w2, a.w_bf16, int64_t(v) * R + r, w);
#pragma unroll
          for (int b = 0; b < MAXB; ++b) {
            if (b >= B) break;
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[b] = fmaf(w[j], e_sm[b * R + r + j], acc[b]);
          }
        }
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
          if (b >= B) break;
          emit(b, v, acc[b], best[b], bidx[b]);
        }
      }
      warp_best<MAXB>(best, bidx, B, sv, si);
    }
    float cv = 0.f;
    int ci = 0;
    warps_best<MAXB, kWarps>(B, sv, si, cv, ci);
    if (int(threadIdx.x) < B) {
      a.cand_v[(int64_t(buf) * G + blockIdx.x) * B + threadIdx.x] = cv;
      a.cand_i[(int64_t(buf) * G + blockIdx.x) * B + threadIdx.x] = ci;
      __threadfence();
    }
    if (!walk_sync(a, gen)) return;
    for (int b = warp; b < B; b += kWarps) {  // every CTA takes the same winner
      float v;
      int ix;
      combine_best(a, buf, b, v, ix);
      if (lane == 0) {
        if (sampled)
          stat_m[b] = v;  // max over the vocabulary of logits / temperature
        else
          prev_s[b] = ix;
      }
    }
    buf ^= 1;
    if (sampled) {
      __syncthreads();
      // softmax denominator: sum of exp(z - max), added over CTAs in CTA order
      float sum[MAXB];
#pragma unroll
      for (int b = 0; b < MAXB; ++b) sum[b] = 0.f;
      for (int v = v0 + threadIdx.x; v < v1; v += THREADS)
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
          if (b >= B) break;
          sum[b] += expf(li_sm[b * a.slice + (v - v0)] / tp - stat_m[b]);
        }
      float bs = 0.f;
      block_sum_b<MAXB, kWarps>(sum, B, sv, bs);
      if (int(threadIdx.x) < B) {
        a.cand_v[(int64_t(buf) * G + blockIdx.x) * B + threadIdx.x] = bs;
        __threadfence();
      }
      if (!walk_sync(a, gen)) return;
      for (int b = warp; b < B; b += kWarps) {
        const float z = combine_sum(a, buf, b);
        if (lane == 0) stat_z[b] = z;
      }
      buf ^= 1;
      __syncthreads();
      // Gumbel-max: argmax of p / (-log(g + 1e-20)), p = exp(z - max) / sum
      float best[MAXB];
      int bidx[MAXB];
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        best[b] = -INFINITY;
        bidx[b] = INT_MAX;
      }
      for (int v = v0 + threadIdx.x; v < v1; v += THREADS)
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
          if (b >= B) break;
          const float p = expf(li_sm[b * a.slice + (v - v0)] / tp - stat_m[b]) / stat_z[b];
          const float g = a.uniforms[(int64_t(i) * B + b) * V + v];
          const float q = p / (-logf(g + 1e-20f));
          if (q > best[b]) {
            best[b] = q;
            bidx[b] = v;
          }
        }
      warp_best<MAXB>(best, bidx, B, sv, si);
      warps_best<MAXB, kWarps>(B, sv, si, cv, ci);
      if (int(threadIdx.x) < B) {
        a.cand_v[(int64_t(buf) * G + blockIdx.x) * B + threadIdx.x] = cv;
        a.cand_i[(int64_t(buf) * G + blockIdx.x) * B + threadIdx.x] = ci;
        __threadfence();
      }
      if (!walk_sync(a, gen)) return;
      for (int b = warp; b < B; b += kWarps) {
        float v;
        int ix;
        combine_best(a, buf, b, v, ix);
        if (lane == 0) prev_s[b] = ix;
      }
      buf ^= 1;
    }
    __syncthreads();  // prev_s[b] was written by the warp that combined row b
    if (int(threadIdx.x) < B) {
      if (prev_s[threadIdx.x] < 0 || prev_s[threadIdx.x] >= V) prev_s[threadIdx.x] = 0;  // all-NaN row
      if (blockIdx.x == 0) a.out_ids[int64_t(threadIdx.x) * (S + 1) + i + 1] = prev_s[threadIdx.x];
    }
    __syncthreads();
  }

  // confidence (CTA 0): hidden half from hc_head_norm plus the Markov half, w1[tok] . wc_r
  if (blockIdx.x == 0 && a.confidence) {
    for (int p = warp; p < B * S; p += kWarps) {
      const int b = p / S, i = p - b * S;
      const int tok = a.out_ids[int64_t(b) * (S + 1) + i];
      float s = 0.f;
      if (a.conf_wr)
        for (int r = lane; r < R; r += 32) s = fmaf(wload(a.w1, a.w_bf16, int64_t(tok) * R + r), a.conf_wr[r], s);
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) a.confidence[p] = (a.conf_part ? a.conf_part[p] : 0.f) + s + a.conf_bias;
    }
  }
}

// Markov head alone (heads.py:26-30): logits[t, v] = w1[ids[t]] . w2[v] (fp32), embed = w1[ids]
__global__ void __launch_bounds__(kWalkThreads) markov_head_kernel(const void* ids, int ids_i64, int64_t n, int vocab,
                                                                   int rank, const void* w1, const void* w2, int w_bf16,
                                                                   float* logits, void* embed) {
  extern __shared__ float e_sm[];  // [rank]
  const int64_t t = blockIdx.y;
  int64_t id = ids_i64 ? static_cast<const int64_t*>(ids)[t] : static_cast<const int32_t*>(ids)[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) raise_device_error(DSM_DEV_ERR_TOKEN_RANGE);
    id = 0;
  }
  for (int r = threadIdx.x; r < rank; r += kWalkThreads) {
    e_sm[r] = wload(w1, w_bf16, id * rank + r);
    if (blockIdx.x == 0 && embed) {
      if (w_bf16)
        static_cast<__nv_bfloat16*>(embed)[t * rank + r] = static_cast<const __nv_bfloat16*>(w1)[id * rank + r];
      else
        static_cast<float*>(embed)[t * rank + r] = static_cast<const float*>(w1)[id * rank + r];
    }
  }
  __syncthreads();
  const int v = blockIdx.x * kWalkThreads + threadIdx.x;
  if (v >= vocab) return;
  float acc = 0.f;
  for (int r = 0; r < rank; r += 8) {
    float w[8];
    wload8(w2, w_bf16, int64_t(v) * rank + r, w);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = fmaf(w[j], e_sm[r + j], acc);
  }
  logits[t * vocab + v] = acc;
}

int walk_ctas(int vocab) {
  return int(std::min<int64_t>(std::min(num_sms(), kWalkCtaBound), ceil_div(vocab, kWalkThreads)));
}

size_t walk_bytes(int batch) { return kWalkHeader + 2 * size_t(2) * kWalkCtaBound * size_t(batch) * 4; }

struct HeadLayout {
  void *y, *xn, *staged, *walk;
  float *conf_part, *xscale, *logits;
  int64_t rows, cap;
  size_t bytes;
};

HeadLayout head_layout(const dsm_head_desc* d, int x_dtype, void* base) {
  HeadLayout L{};
  const int64_t n = d->batch * d->block;
  const size_t es = x_dtype == DSM_DT_BF16 ? 2 : 4;
  L.rows = x_dtype == DSM_DT_BF16 ? n : 2 * n;
  L.cap = dsm_stage_rows_cap(L.rows);
  char* p = static_cast<char*>(base);
  size_t off = 0;
  auto take = [&](size_t b) {
    void* q = p ? p + off : nullptr;
    off += (b + 255) / 256 * 256;
    return q;
  };
  L.y = take(size_t(n) * d->dim * es);
  L.xn = take(size_t(n) * d->dim * es);
  L.conf_part = static_cast<float*>(take(size_t(n) * 4));
  L.staged = take(dsm_stage_bytes(L.cap, d->dim));
  L.xscale = static_cast<float*>(take(size_t(L.cap) * 4));
  L.logits = static_cast<float*>(take(size_t(L.rows) * d->vocab * 4));
  L.walk = take(walk_bytes(int(d->batch)));
  L.bytes = off;
  return L;
}

int check_markov(int vocab, int rank, int w_dtype, const void* w1, const void* w2) {
  DSM_REQUIRE(vocab > 0 && rank > 0 && rank % 8 == 0, "draft head: rank must be a positive multiple of 8");
  DSM_REQUIRE(w_dtype == DSM_DT_F32 || w_dtype == DSM_DT_BF16, "draft head: Markov tables must be F32 or BF16");
  DSM_REQUIRE(w1 && w2, "draft head: NULL Markov table");
  DSM_REQUIRE((reinterpret_cast<uintptr_t>(w2) & 15) == 0, "draft head: markov_w2 must be 16-byte aligned");
  return DSM_OK;
}

int launch_walk(const WalkArgs& a0, void* walk_ws, cudaStream_t s) {
  WalkArgs a = a0;
  const int G = walk_ctas(a.vocab);
  a.slice = int(ceil_div(a.vocab, G));
  char* w = static_cast<char*>(walk_ws);
  a.bar = reinterpret_cast<unsigned*>(w);
  a.abort_flag = reinterpret_cast<int*>(w + 8);
  a.cand_v = reinterpret_cast<float*>(w + kWalkHeader);
  a.cand_i = reinterpret_cast<int*>(w + kWalkHeader + 2 * size_t(kWalkCtaBound) * a.batch * 4);
  if (cudaMemsetAsync(w, 0, kWalkHeader, s) != cudaSuccess) return check_launch("draft head walk reset");
  const int maxb = a.batch <= 8 ? 8 : 32;
  const size_t smem =
      (size_t(walk_e_floats(a.batch, a.rank, maxb)) + (a.temperature > 0.f ? size_t(a.batch) * a.slice : 0)) * 4;
  void* args[] = {&a};
  auto go = [&](auto kern, int threads) {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
      return check_launch("draft head walk smem attribute");
    if (cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kern), dim3(G), dim3(threads), args, smem, s) !=
        cudaSuccess)
      return check_launch("draft head walk (cooperative launch)");
    return check_launch("draft head walk");
  };
  // up to 8 batch rows: 16 warps per CTA (128 registers each), twice the Markov-row and logit
  // loads in flight of 8 warps, which left the walk waiting on L2; the 32-row form needs its
  // registers at 8 warps
  if (a.batch <= 8) return go(head_walk_kernel<8, 512>, 512);
  return go(head_walk_kernel<32, 256>, 256);
}

}  // namespace
}  // namespace dsm

using namespace dsm;

extern "C" int dsm_markov_head(const void* ids, int ids_dtype, int64_t n, int vocab, int rank, const void* w1,
                               const void* w2, int w_dtype, float* logits, void* embed, void* stream) {
  if (int rc = check_markov(vocab, rank, w_dtype, w1, w2)) return rc;
  DSM_REQUIRE(n >= 0 && n <= 65535, "dsm_markov_head: n must be in [0, 65535]");
  DSM_REQUIRE(ids_dtype == DSM_DT_I32 || ids_dtype == DSM_DT_I64, "dsm_markov_head: ids must be I32 or I64");
  if (n == 0) return DSM_OK;
  DSM_REQUIRE(ids && logits, "dsm_markov_head: NULL pointer");
  const dim3 grid(unsigned(ceil_div(vocab, kWalkThreads)), unsigned(n));
  markov_head_kernel<<<grid, kWalkThreads, size_t(rank) * 4, as_stream(stream)>>>(
      ids, ids_dtype == DSM_DT_I64, n, vocab, rank, w1, w2, w_dtype == DSM_DT_BF16, logits, embed);
  return check_launch("markov_head");
}

extern "C" size_t dsm_draft_head_workspace_bytes(const dsm_head_desc* d, int x_dtype) {
  if (!d || d->batch <= 0 || d->block <= 0 || d->dim <= 0 || d->vocab <= 0) return 0;
  return head_layout(d, x_dtype, nullptr).bytes;
}

extern "C" int dsm_draft_head(const dsm_head_desc* d, const void* x, int x_dtype, const void* anchor, int anchor_dtype,
                              float temperature, const float* uniforms, int32_t* out_ids, float* biased_logits,
                              float* confidence, void* y_out, void* workspace, size_t workspace_bytes, void* stream) {
  DSM_REQUIRE(d, "dsm_draft_head: NULL descriptor");
  DSM_REQUIRE(d->batch > 0 && d->batch <= 32 && d->block > 0 && d->dim > 0 && d->vocab > 0,
              "dsm_draft_head: bad shape (batch must be 1..32)");
  DSM_REQUIRE(x_dtype == DSM_DT_F32 || x_dtype == DSM_DT_BF16, "dsm_draft_head: x must be F32 or BF16");
  DSM_REQUIRE(anchor_dtype == DSM_DT_I32 || anchor_dtype == DSM_DT_I64, "dsm_draft_head: anchor must be I32 or I64");
  DSM_REQUIRE(temperature >= 0.f, "dsm_draft_head: temperature must be >= 0");
  DSM_REQUIRE(temperature == 0.f || uniforms, "dsm_draft_head: sampling above temperature 0 needs uniforms");
  DSM_REQUIRE(x && anchor && out_ids && biased_logits && d->head_w && d->hc_fn && d->hc_scale && d->hc_base,
              "dsm_draft_head: NULL pointer");
  if (int rc = check_markov(d->vocab, d->rank, d->markov_dtype, d->markov_w1, d->markov_w2)) return rc;
  const HeadLayout L = head_layout(d, x_dtype, workspace);
  if (!workspace || workspace_bytes < L.bytes) return fail(DSM_ERR_WORKSPACE, "dsm_draft_head: workspace too small");
  cudaStream_t s = as_stream(stream);
  const int64_t n = d->batch * d->block;
  void* y = y_out ? y_out : L.y;
  int rc = dsm_hc_head_norm(x, x_dtype, n, d->hc_mult, d->dim, d->hc_fn, d->hc_scale, d->hc_base, d->norm_eps,
                            d->hc_eps, d->norm_weight, d->conf_w, y, L.xn, L.conf_part, stream);
  if (rc) return rc;
  if (x_dtype == DSM_DT_BF16)
    rc = dsm_stage_rows(L.xn, DSM_DT_BF16, n, d->dim, nullptr, n, 1, L.staged, L.cap, L.xscale, stream);
  else
    rc = stage_rows_hilo(static_cast<const float*>(L.xn), n, d->dim, L.staged, L.cap, L.xscale, stream);
  if (rc) return rc;
  rc = dsm_linear(L.staged, L.xscale, L.cap, d->dim, d->head_wfmt, d->head_group_size, d->head_w, d->vocab, L.logits,
                  d->vocab, L.rows, stream);
  if (rc) return rc;
  WalkArgs a{};
  a.logits = L.logits;
  a.lo_offset = x_dtype == DSM_DT_BF16 ? 0 : n;
  a.batch = int(d->batch);
  a.block = d->block;
  a.vocab = d->vocab;
  a.rank = d->rank;
  a.w1 = d->markov_w1;
  a.w2 = d->markov_w2;
  a.w_bf16 = d->markov_dtype == DSM_DT_BF16;
  a.anchor = anchor;
  a.anchor_i64 = anchor_dtype == DSM_DT_I64;
  a.temperature = temperature;
  a.uniforms = uniforms;
  a.conf_part = d->conf_w ? L.conf_part : nullptr;
  a.conf_wr = d->conf_w ? d->conf_w + d->dim : nullptr;
  a.conf_bias = d->conf_bias;
  a.out_ids = out_ids;
  a.biased = biased_logits;
  a.confidence = confidence;
  return launch_walk(a, L.walk, s);
}
