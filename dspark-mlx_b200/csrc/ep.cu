// Expert-parallel plumbing kernels: the row gather a rank sends to the owners of its
// routed experts, and the local expert id of every row it receives. The exchange itself
// (per-expert counts, then rows, then results) runs on NCCL all-to-all from the host.
#include <algorithm>

#include "common.cuh"

namespace dsm {
namespace {

template <typename T>
__global__ void __launch_bounds__(128) gather_rows_kernel(const T* __restrict__ x, int64_t n_tokens, int dim,
                                                          const int32_t* __restrict__ perm, int topk,
                                                          T* __restrict__ out) {
  const int64_t r = blockIdx.x;
  int64_t t = perm ? int64_t(perm[r]) / topk : r;
  if (t < 0 || t >= n_tokens) {
    if (threadIdx.x == 0) raise_device_error(DSM_DEV_ERR_TOKEN_RANGE);
    t = 0;
  }
  const T* src = x + t * dim;
  T* dst = out + r * dim;
  const int bytes = dim * int(sizeof(T));
  if ((bytes & 15) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) d4[i] = s4[i];
  } else {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) dst[i] = src[i];
  }
}

constexpr int kSegMax = 4096;

__global__ void __launch_bounds__(1024) segment_ids_kernel(const int32_t* __restrict__ counts, int n_segments,
                                                           int e_local, int32_t* __restrict__ ids, int64_t n_rows) {
  __shared__ int32_t start[kSegMax + 1];
  __shared__ int32_t wsum[32];
  // exclusive scan of the counts (up to 4 per thread)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int v[4], tot = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int s = tid * 4 + i;
    v[i] = s < n_segments ? counts[s] : 0;
    tot += v[i];
  }
  int incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    wsum[lane] = w;
  }
  __syncthreads();
  int run = incl - tot + (warp ? wsum[warp - 1] : 0);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int s = tid * 4 + i;
    if (s <= kSegMax) start[s] = run;
    run += v[i];
  }
  __syncthreads();
  for (int64_t r = blockIdx.x * int64_t(blockDim.x) + tid; r < n_rows; r += int64_t(gridDim.x) * blockDim.x) {
    // largest segment s with start[s] <= r
    int lo = 0, hi = n_segments - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (start[mid] <= r)
        lo = mid;
      else
        hi = mid - 1;
    }
    ids[r] = lo % e_local;
  }
}

}  // namespace
}  // namespace dsm

extern "C" int dsm_gather_rows(const void* x, int x_dtype, int64_t n_tokens, int dim, const int32_t* perm,
                               int64_t n_rows, int topk, void* out, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(dim > 0 && n_rows >= 0 && n_tokens >= 0 && n_rows < (int64_t(1) << 31), "dsm_gather_rows: bad shape");
  DSM_REQUIRE(x_dtype == DSM_DT_F32 || x_dtype == DSM_DT_BF16, "dsm_gather_rows: x must be F32 or BF16");
  DSM_REQUIRE(!perm || topk >= 1, "dsm_gather_rows: topk must be >= 1 with a permutation");
  if (n_rows == 0) return DSM_OK;
  DSM_REQUIRE(x && out, "dsm_gather_rows: NULL pointer");
  cudaStream_t s = as_stream(stream);
  if (x_dtype == DSM_DT_BF16)
    gather_rows_kernel<uint16_t><<<unsigned(n_rows), 128, 0, s>>>(static_cast<const uint16_t*>(x), n_tokens, dim,
                                                                  perm, topk, static_cast<uint16_t*>(out));
  else
    gather_rows_kernel<float><<<unsigned(n_rows), 128, 0, s>>>(static_cast<const float*>(x), n_tokens, dim, perm,
                                                               topk, static_cast<float*>(out));
  return check_launch("gather_rows");
}

extern "C" int dsm_segment_ids(const int32_t* counts, int n_segments, int e_local, int32_t* ids, int64_t n_rows,
                               void* stream) {
  using namespace dsm;
  DSM_REQUIRE(n_segments >= 1 && n_segments <= kSegMax, "dsm_segment_ids: n_segments must be in [1, 4096]");
  DSM_REQUIRE(e_local >= 1 && n_segments % e_local == 0, "dsm_segment_ids: n_segments must be a multiple of e_local");
  DSM_REQUIRE(n_rows >= 0, "dsm_segment_ids: bad n_rows");
  if (n_rows == 0) return DSM_OK;
  DSM_REQUIRE(counts && ids, "dsm_segment_ids: NULL pointer");
  const unsigned blocks = unsigned(std::min<int64_t>(ceil_div(n_rows, 1024), 64));
  segment_ids_kernel<<<blocks, 1024, 0, as_stream(stream)>>>(counts, n_segments, e_local, ids, n_rows);
  return check_launch("segment_ids");
}
