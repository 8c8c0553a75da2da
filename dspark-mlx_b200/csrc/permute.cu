// Token permutation: per-expert counts, offsets and the stable expert-sorted order of the
// flattened (token, slot) routing pairs.
//
// The reference never materialises these: gather_mm takes the unsorted per-(token, slot)
// expert ids (dspark_mlx/model/moe.py:145-148). Sorting the pairs by expert lets every
// expert's weights be streamed once per call instead of once per (token, slot).
//
//   1. block_hist     each 1024-pair block histograms its expert ids (shared atomics)
//   2. scan           per expert: base of every block (exclusive over blocks), counts,
//                     offsets (exclusive scan over experts)
//   3. scatter        each pair's sorted position = block base + pairs of the same expert
//                     in earlier warps of the block + earlier lanes of its warp
//                     (__match_any_sync); stable by construction.
#include "common.cuh"

namespace dsm {
namespace {

constexpr int kPermBlock = 1024;

__global__ void __launch_bounds__(kPermBlock) block_hist_kernel(const int32_t* __restrict__ idx, int64_t n_pairs,
                                                                int n_experts, int32_t* __restrict__ hist) {
  extern __shared__ int32_t sh[];
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int64_t i = int64_t(blockIdx.x) * kPermBlock + threadIdx.x;
  if (i < n_pairs) {
    const int e = idx[i];
    if (e >= 0 && e < n_experts)
      atomicAdd(&sh[e], 1);
    else
      raise_device_error(DSM_DEV_ERR_EXPERT_RANGE);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) hist[int64_t(blockIdx.x) * n_experts + e] = sh[e];
}

// one block; thread e owns expert e (loops if E > blockDim)
__global__ void __launch_bounds__(1024) scan_kernel(int32_t* __restrict__ hist, int n_blocks, int n_experts,
                                                    int32_t* __restrict__ counts, int32_t* __restrict__ offsets) {
  extern __shared__ int32_t tot[];  // [n_experts]
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) {
    int32_t run = 0;
    for (int b = 0; b < n_blocks; ++b) {
      const int32_t h = hist[int64_t(b) * n_experts + e];
      hist[int64_t(b) * n_experts + e] = run;  // exclusive within the expert
      run += h;
    }
    tot[e] = run;
    counts[e] = run;
  }
  __syncthreads();
  // exclusive scan over experts (serial per 32-chunk is plenty for E <= 1024)
  if (threadIdx.x == 0) {
    int32_t acc = 0;
    for (int e = 0; e < n_experts; ++e) {
      const int32_t c = tot[e];
      tot[e] = acc;
      acc += c;
    }
    offsets[n_experts] = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) {
    offsets[e] = tot[e];
    for (int b = 0; b < n_blocks; ++b) hist[int64_t(b) * n_experts + e] += tot[e];
  }
}

__global__ void __launch_bounds__(kPermBlock) scatter_kernel(const int32_t* __restrict__ idx, int64_t n_pairs,
                                                             int n_experts, const int32_t* __restrict__ base,
                                                             int32_t* __restrict__ perm, int32_t* __restrict__ inv) {
  extern __shared__ int32_t wh[];  // [32 warps][n_experts]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = int64_t(blockIdx.x) * kPermBlock + threadIdx.x;
  int e = -1;
  if (i < n_pairs) {
    e = idx[i];
    if (e < 0 || e >= n_experts) e = -1;
  }
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  // wh[w][e] = pairs of expert e in warp w of this block
  for (int k = threadIdx.x; k < 32 * n_experts; k += blockDim.x) wh[k] = 0;
  __syncthreads();
  if (e >= 0 && rank == 0) wh[warp * n_experts + e] = __popc(peers);
  __syncthreads();
  if (e >= 0) {
    int pos = base[int64_t(blockIdx.x) * n_experts + e] + rank;
    for (int w = 0; w < warp; ++w) pos += wh[w * n_experts + e];
    perm[pos] = int32_t(i);
    inv[i] = pos;
  } else if (i < n_pairs) {
    inv[i] = 0;
  }
}

// Decode-sized inputs: the whole permutation in one CTA (histogram, scan, then a stable
// scatter of 1024-pair chunks with running per-expert cursors).
constexpr int64_t kSmallPairs = 16384;

__global__ void __launch_bounds__(kPermBlock) permute_small_kernel(const int32_t* __restrict__ idx, int64_t n_pairs,
                                                                   int n_experts, int32_t* __restrict__ counts,
                                                                   int32_t* __restrict__ offsets,
                                                                   int32_t* __restrict__ perm,
                                                                   int32_t* __restrict__ inv) {
  extern __shared__ int32_t sm[];
  int32_t* cursor = sm;                  // [n_experts]
  int32_t* wsum = sm + n_experts;        // [32]
  int32_t* wh = wsum + 32;               // [32][n_experts]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int k = tid; k < n_experts; k += kPermBlock) cursor[k] = 0;
  for (int k = tid; k < 32 * n_experts; k += kPermBlock) wh[k] = 0;
  __syncthreads();
  for (int64_t i = tid; i < n_pairs; i += kPermBlock) {
    const int e = idx[i];
    if (e >= 0 && e < n_experts)
      atomicAdd(&cursor[e], 1);
    else
      raise_device_error(DSM_DEV_ERR_EXPERT_RANGE);
  }
  __syncthreads();
  // exclusive scan of the counts (n_experts <= 1024: one expert per thread)
  const int c = tid < n_experts ? cursor[tid] : 0;
  int v = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) wsum[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int wv = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wv, o);
      if (lane >= o) wv += t;
    }
    wsum[lane] = wv;  // inclusive over warps
  }
  __syncthreads();
  const int excl = v - c + (warp > 0 ? wsum[warp - 1] : 0);
  if (tid < n_experts) {
    counts[tid] = c;
    offsets[tid] = excl;
    cursor[tid] = excl;
  }
  if (tid == 0) offsets[n_experts] = wsum[31];
  __syncthreads();
  for (int64_t base = 0; base < n_pairs; base += kPermBlock) {
    const int64_t i = base + tid;
    int e = -1;
    if (i < n_pairs) {
      e = idx[i];
      if (e < 0 || e >= n_experts) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wh[warp * n_experts + e] = __popc(peers);
    __syncthreads();
    if (e >= 0) {
      int pos = cursor[e] + rank;
      for (int w = 0; w < warp; ++w) pos += wh[w * n_experts + e];
      perm[pos] = int32_t(i);
      inv[i] = pos;
    } else if (i < n_pairs) {
      inv[i] = 0;
    }
    __syncthreads();
    for (int k = tid; k < n_experts; k += kPermBlock) {
      int add = 0;
      for (int w = 0; w < 32; ++w) {
        add += wh[w * n_experts + k];
        wh[w * n_experts + k] = 0;
      }
      cursor[k] += add;
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace dsm

extern "C" size_t dsm_permute_workspace_bytes(int64_t n_pairs, int n_experts) {
  const int64_t blocks = dsm::ceil_div(n_pairs > 0 ? n_pairs : 1, dsm::kPermBlock);
  return size_t(blocks) * size_t(n_experts) * sizeof(int32_t);
}

extern "C" int dsm_permute(const int32_t* indices, int64_t n_pairs, int n_experts, int32_t* counts,
                           int32_t* offsets, int32_t* perm, int32_t* inv, void* workspace, size_t workspace_bytes,
                           void* stream) {
  using namespace dsm;
  DSM_REQUIRE(n_pairs >= 0 && n_pairs < (int64_t(1) << 31), "dsm_permute: n_pairs out of range");
  DSM_REQUIRE(n_experts > 0 && n_experts <= 1024, "dsm_permute: n_experts must be in [1, 1024]");
  DSM_REQUIRE(counts && offsets && (n_pairs == 0 || (indices && perm && inv && workspace)),
              "dsm_permute: NULL pointer");
  if (workspace_bytes < dsm_permute_workspace_bytes(n_pairs, n_experts))
    return fail(DSM_ERR_WORKSPACE, "dsm_permute: workspace too small");
  cudaStream_t s = as_stream(stream);
  if (n_pairs > 0 && n_pairs <= kSmallPairs) {
    const size_t sm = size_t(n_experts + 32 + 32 * n_experts) * sizeof(int32_t);
    if (sm > 48 * 1024 &&
        cudaFuncSetAttribute(permute_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)) != cudaSuccess)
      return check_launch("permute_small smem attribute");
    permute_small_kernel<<<1, kPermBlock, sm, s>>>(indices, n_pairs, n_experts, counts, offsets, perm, inv);
    return check_launch("permute_small");
  }
  const int blocks = int(ceil_div(n_pairs > 0 ? n_pairs : 1, kPermBlock));
  int32_t* hist = static_cast<int32_t*>(workspace);
  const size_t wh_bytes = size_t(32) * n_experts * sizeof(int32_t);
  if (wh_bytes > 48 * 1024 &&
      cudaFuncSetAttribute(scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(wh_bytes)) != cudaSuccess)
    return check_launch("scatter smem attribute");
  if (n_pairs > 0) {
    block_hist_kernel<<<blocks, kPermBlock, n_experts * sizeof(int32_t), s>>>(indices, n_pairs, n_experts, hist);
    if (int rc = check_launch("block_hist")) return rc;
  } else {
    if (cudaMemsetAsync(hist, 0, size_t(n_experts) * sizeof(int32_t), s) != cudaSuccess)
      return check_launch("memset");
  }
  scan_kernel<<<1, 1024, n_experts * sizeof(int32_t), s>>>(hist, blocks, n_experts, counts, offsets);
  if (int rc = check_launch("scan")) return rc;
  if (n_pairs == 0) return DSM_OK;
  scatter_kernel<<<blocks, kPermBlock, wh_bytes, s>>>(indices, n_pairs, n_experts, hist, perm, inv);
  return check_launch("scatter");
}
