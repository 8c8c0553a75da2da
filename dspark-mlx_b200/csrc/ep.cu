// Row gather (the draft block's embedding rows) and the expert-parallel exchange.
//
// Expert parallelism (no counterpart in the reference, which runs on one device:
// tests/reference_model.py:55-56): rank r of W owns experts [r * El, (r + 1) * El). Every rank
// holds one exchange buffer that its peers map (CUDA IPC) and write into with plain stores
// over NVLink; nothing in a step waits on the host:
//
//   dispatch  each (token, slot) row goes straight into its owner's buffer, in the sender's
//             expert-sorted order (block [set][sender]), with the sender's per-expert counts;
//             the last CTA to finish raises the sender's epoch flag in every peer;
//   receive   one CTA waits (bounded) for every sender's flag, then lays the arrived rows out
//             by local expert: offsets [El + 1], the staging permutation and the row count;
//   return    each result row goes back into its sender's buffer at the slot it came from;
//             the last CTA raises this rank's result flag in every peer;
//   wait      (bounded) for every owner's result flag; the weighted combine then reads the
//             results through the row map the dispatch wrote.
//
// Two buffer sets alternate by step (epoch & 1): a rank can only start step e + 2 after it
// has the results of step e + 1 from every peer, which every peer produces after it finished
// reading step e's rows, so a set is never overwritten while it is read. Flags hold the epoch
// of the step that raised them, so they never need clearing. Every wait gives up after ~2 s
// of wall time, records DSM_DEV_ERR_PEER_TIMEOUT and lets the step finish (on zero rows).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

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


constexpr int kEpCopyThreads = 128;
constexpr int kEpMaxWorld = 64;
constexpr uint64_t kEpWaitNs = 2000000000ull;

struct EpGeom {
  int world, rank, e_local, dim, elem;  // elem: bytes per activation element
  int64_t cap;                          // rows per (sender, owner) block
  int64_t off_rows, off_counts, off_rflags, off_back, off_bflags;
};

__host__ __device__ inline int64_t ep_round(int64_t v) { return (v + 255) / 256 * 256; }

__host__ __device__ inline EpGeom ep_geom(int world, int rank, int e_local, int dim, int elem, int64_t cap) {
  EpGeom g{world, rank, e_local, dim, elem, cap, 0, 0, 0, 0, 0};
  int64_t o = 0;
  g.off_rows = o;
  o += ep_round(2 * int64_t(world) * cap * dim * elem);
  g.off_counts = o;
  o += ep_round(2 * int64_t(world) * e_local * 4);
  g.off_rflags = o;
  o += ep_round(2 * int64_t(world) * 4);
  g.off_back = o;
  o += ep_round(2 * int64_t(world) * cap * dim * 4);
  g.off_bflags = o;
  return g;
}
inline int64_t ep_bytes(const EpGeom& g) { return g.off_bflags + ep_round(2 * int64_t(g.world) * 4); }

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Spin until *flag == epoch, for at most ~2 s; false (and the device error word) on timeout.
__device__ __forceinline__ bool ep_wait_flag(const uint32_t* flag, uint32_t epoch) {
  if (ld_acquire_sys(flag) == epoch) return true;
  const uint64_t t0 = global_timer_ns();
  while (ld_acquire_sys(flag) != epoch) {
    if (global_timer_ns() - t0 > kEpWaitNs) {
      raise_device_error(DSM_DEV_ERR_PEER_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Copies `bytes` (a multiple of 16, both ends 16-byte aligned) with the CTA's threads.
// One row by the CTA, four 16-byte loads per thread in flight before their stores.
__device__ __forceinline__ void copy_row16(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, int bytes) {
  const int n = bytes / 16;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  for (int i0 = threadIdx.x; i0 < n; i0 += 4 * blockDim.x) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * int(blockDim.x);
      if (i < n) v[u] = s4[i];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * int(blockDim.x);
      if (i < n) d4[i] = v[u];
    }
  }
}

// The CTA that finishes last raises `flag_off` (+ 4 * index) in every peer's buffer. Every
// thread's peer stores are fenced at system scope before its CTA counts itself done.
__device__ __forceinline__ void ep_signal_peers(const uint64_t* peer_base, int world, int64_t flag_off,
                                                uint32_t* done, uint32_t epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < world; ++d)
        st_release_sys(reinterpret_cast<uint32_t*>(peer_base[d] + flag_off), epoch);
      *done = 0;  // ready for the next launch (stream-ordered after this one)
    }
  }
}

// grid = min(n_pairs, kEpDispatchCtas) + 1 CTAs: CTA b < grid - 1 sends sorted rows b,
// b + grid - 1, ...; the last one sends the counts. A few CTAs per SM that each loop over
// rows keep the NVLink stores flowing, and the system-scope fence and the completion count
// are paid once per CTA, not once per row.
constexpr int64_t kEpDispatchCtas = 1024;
__global__ void __launch_bounds__(kEpCopyThreads) ep_dispatch_kernel(
    EpGeom g, const uint8_t* __restrict__ x, int64_t n_tokens, const int32_t* __restrict__ indices,
    const int32_t* __restrict__ perm, const int32_t* __restrict__ offsets, const int32_t* __restrict__ counts,
    int64_t n_pairs, int topk, const uint64_t* __restrict__ peer_base, int32_t* __restrict__ row_map,
    uint32_t* done, uint32_t epoch) {
  const int set = int(epoch & 1u);
  const int64_t row_ctas = int64_t(gridDim.x) - 1;
  // The sorted rows go out in owner order, starting at owner rank + 1: at any moment the
  // ranks' CTAs store into different owners instead of all into owner 0, then all into 1...
  const int64_t start = n_pairs > 0 ? offsets[((g.rank + 1) % g.world) * g.e_local] : 0;
  for (int64_t k = blockIdx.x; k < n_pairs && int64_t(blockIdx.x) < row_ctas; k += row_ctas) {
    const int64_t i = k + start < n_pairs ? k + start : k + start - n_pairs;
    const int32_t pair = perm[i];
    const int e = (pair >= 0 && pair < n_pairs) ? indices[pair] : -1;
    const int d = e >= 0 ? e / g.e_local : -1;
    const int64_t j = d >= 0 && d < g.world ? int64_t(i) - offsets[d * g.e_local] : -1;
    const int64_t t = pair / topk;
    if (d < 0 || d >= g.world || j < 0 || j >= g.cap || t >= n_tokens) {
      if (threadIdx.x == 0) {
        raise_device_error(d < 0 || d >= g.world ? DSM_DEV_ERR_EXPERT_RANGE : DSM_DEV_ERR_CAPACITY);
        if (pair >= 0 && pair < n_pairs) row_map[pair] = 0;  // the combine reads an in-range row
      }
    } else {
      const int64_t row_bytes = int64_t(g.dim) * g.elem;
      uint8_t* dst = reinterpret_cast<uint8_t*>(peer_base[d]) + g.off_rows +
                     ((int64_t(set) * g.world + g.rank) * g.cap + j) * row_bytes;
      copy_row16(dst, x + t * row_bytes, int(row_bytes));
      if (threadIdx.x == 0) row_map[pair] = int32_t(d * g.cap + j);
    }
  }
  if (int64_t(blockIdx.x) == row_ctas) {
    for (int c = threadIdx.x; c < g.world * g.e_local; c += blockDim.x) {
      const int d = c / g.e_local, e = c % g.e_local;
      int32_t* dst = reinterpret_cast<int32_t*>(peer_base[d] + g.off_counts) +
                     (int64_t(set) * g.world + g.rank) * g.e_local + e;
      *dst = counts[c];
    }
  }
  ep_signal_peers(peer_base, g.world, g.off_rflags + (int64_t(set) * g.world + g.rank) * 4, done, epoch);
}

// One CTA: waits for every sender, then the local layout of the arrived rows:
//   offsets[e] (El + 1)  rows of local experts < e, over all senders;
//   lperm[p]             arrival row (sender * cap + slot) of staged position p, positions
//                        grouped by local expert, senders ascending, each sender's order kept;
//   n_valid[0]           rows arrived; n_valid[1 + s] rows from sender s.
__global__ void __launch_bounds__(1024) ep_receive_kernel(EpGeom g, const uint8_t* own, uint32_t epoch,
                                                          int32_t* __restrict__ offsets, int32_t* __restrict__ lperm,
                                                          int32_t* __restrict__ n_valid) {
  extern __shared__ int32_t ep_sm[];
  const int W = g.world, El = g.e_local, tid = threadIdx.x;
  const int set = int(epoch & 1u);
  int32_t* cnt = ep_sm;              // [W][El]
  int32_t* src_pos = cnt + W * El;   // [W][El]: rows of the sender's earlier experts
  int32_t* before = src_pos + W * El;  // [W][El]: rows of earlier senders for expert e
  int32_t* off = before + W * El;    // [El + 1]
  __shared__ int ok_all;
  if (tid == 0) ok_all = 1;
  __syncthreads();
  if (tid < W) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(own + g.off_rflags) + int64_t(set) * W + tid;
    if (!ep_wait_flag(f, epoch)) atomicAnd(&ok_all, 0);
  }
  __syncthreads();
  const int32_t* rc = reinterpret_cast<const int32_t*>(own + g.off_counts) + int64_t(set) * W * El;
  for (int c = tid; c < W * El; c += blockDim.x) {
    int32_t v = ok_all ? int32_t(ld_acquire_sys(reinterpret_cast<const uint32_t*>(rc + c))) : 0;
    cnt[c] = (v < 0 || v > g.cap) ? 0 : v;
  }
  __syncthreads();
  for (int s = tid; s < W; s += blockDim.x) {  // a sender's rows fit its block, or none is used
    int64_t run = 0;
    for (int e = 0; e < El; ++e) run += cnt[s * El + e];
    if (run > g.cap) {
      raise_device_error(DSM_DEV_ERR_CAPACITY);
      for (int e = 0; e < El; ++e) cnt[s * El + e] = 0;
    }
  }
  __syncthreads();
  for (int s = tid; s < W; s += blockDim.x) {  // prefix within each sender's block
    int run = 0;
    for (int e = 0; e < El; ++e) {
      src_pos[s * El + e] = run;
      run += cnt[s * El + e];
    }
    n_valid[1 + s] = run;
  }
  for (int e = tid; e < El; e += blockDim.x) {  // prefix over senders for each expert
    int run = 0;
    for (int s = 0; s < W; ++s) {
      before[s * El + e] = run;
      run += cnt[s * El + e];
    }
    off[e] = run;  // total of expert e, scanned below
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int e = 0; e < El; ++e) {
      const int v = off[e];
      off[e] = run;
      run += v;
    }
    off[El] = run;
    n_valid[0] = run;
  }
  __syncthreads();
  for (int e = tid; e <= El; e += blockDim.x) offsets[e] = off[e];
  for (int c = tid; c < W * El; c += blockDim.x) {
    const int s = c / El, e = c % El;
    const int base = off[e] + before[c];
    const int32_t src = int32_t(int64_t(s) * g.cap + src_pos[c]);
    for (int j = 0; j < cnt[c]; ++j) lperm[base + j] = src + j;
  }
}

// grid = W * per CTAs: CTA b serves sender s = (b + rank + 1) % W (so the CTAs that start
// first store into every sender, each rank beginning with a different one) and sends rows
// q = c, c + per, ... (c = b / W) of the rows that arrived from s (arrival row s * cap + q)
// back to s, at slot q. per = kEpReturnCtas / W (at least 32): about as many CTAs in all as
// the dispatch uses, whatever the world size.
constexpr int kEpReturnCtas = 1024;
inline int ep_return_per_sender(int world) { return std::max(32, kEpReturnCtas / world); }
__global__ void __launch_bounds__(kEpCopyThreads) ep_return_kernel(EpGeom g, const float* __restrict__ o_rows,
                                                                   const int32_t* __restrict__ n_valid,
                                                                   const uint64_t* __restrict__ peer_base,
                                                                   uint32_t* done, uint32_t epoch, int per) {
  const int set = int(epoch & 1u);
  const int s = (int(blockIdx.x) + g.rank + 1) % g.world;
  const int64_t row_bytes = int64_t(g.dim) * 4;
  uint8_t* dst0 = reinterpret_cast<uint8_t*>(peer_base[s]) + g.off_back +
                  (int64_t(set) * g.world + g.rank) * g.cap * row_bytes;
  const int64_t n = n_valid[1 + s];
  for (int64_t q = blockIdx.x / g.world; q < n; q += per)
    copy_row16(dst0 + q * row_bytes, reinterpret_cast<const uint8_t*>(o_rows + (int64_t(s) * g.cap + q) * g.dim),
               int(row_bytes));
  ep_signal_peers(peer_base, g.world, g.off_bflags + (int64_t(set) * g.world + g.rank) * 4, done, epoch);
}

__global__ void ep_wait_results_kernel(EpGeom g, const uint8_t* own, uint32_t epoch) {
  const int set = int(epoch & 1u);
  if (int(threadIdx.x) < g.world)
    ep_wait_flag(reinterpret_cast<const uint32_t*>(own + g.off_bflags) + int64_t(set) * g.world + threadIdx.x, epoch);
}

EpGeom geom_of(const dsm_ep_desc* d) {
  return ep_geom(d->world, d->rank, d->e_local, d->dim, d->x_dtype == DSM_DT_BF16 ? 2 : 4, d->capacity);
}

int check_desc(const dsm_ep_desc* d, const char* who) {
  DSM_REQUIRE(d != nullptr, std::string(who) + ": desc is NULL");
  DSM_REQUIRE(d->world >= 1 && d->world <= kEpMaxWorld && d->rank >= 0 && d->rank < d->world,
              std::string(who) + ": bad world / rank");
  DSM_REQUIRE(d->e_local >= 1 && int64_t(d->e_local) * d->world <= 4096, std::string(who) + ": bad e_local");
  DSM_REQUIRE(d->dim > 0 && d->capacity >= 1 && d->capacity < (int64_t(1) << 24), std::string(who) + ": bad shape");
  DSM_REQUIRE(d->x_dtype == DSM_DT_BF16 || d->x_dtype == DSM_DT_F32, std::string(who) + ": x must be BF16 or F32");
  DSM_REQUIRE((int64_t(d->dim) * (d->x_dtype == DSM_DT_BF16 ? 2 : 4)) % 16 == 0,
              std::string(who) + ": rows must be a multiple of 16 bytes");
  return DSM_OK;
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

extern "C" size_t dsm_ep_buffer_bytes(const dsm_ep_desc* d) {
  if (dsm::check_desc(d, "dsm_ep_buffer_bytes") != DSM_OK) return 0;
  return size_t(dsm::ep_bytes(dsm::geom_of(d)));
}

extern "C" int64_t dsm_ep_rows_offset(const dsm_ep_desc* d, uint32_t epoch) {
  if (dsm::check_desc(d, "dsm_ep_rows_offset") != DSM_OK) return -1;
  const dsm::EpGeom g = dsm::geom_of(d);
  return g.off_rows + int64_t(epoch & 1u) * g.world * g.cap * g.dim * g.elem;
}

extern "C" int64_t dsm_ep_results_offset(const dsm_ep_desc* d, uint32_t epoch) {
  if (dsm::check_desc(d, "dsm_ep_results_offset") != DSM_OK) return -1;
  const dsm::EpGeom g = dsm::geom_of(d);
  return g.off_back + int64_t(epoch & 1u) * g.world * g.cap * g.dim * 4;
}

extern "C" int dsm_ep_dispatch(const dsm_ep_desc* d, const void* x, int64_t n_tokens, const int32_t* indices,
                               const int32_t* perm, const int32_t* offsets, const int32_t* counts, int topk,
                               const uint64_t* peer_base, int32_t* row_map, uint32_t* done, uint32_t epoch,
                               void* stream) {
  using namespace dsm;
  if (int rc = check_desc(d, "dsm_ep_dispatch")) return rc;
  DSM_REQUIRE(n_tokens >= 0 && topk >= 1 && n_tokens * topk < (int64_t(1) << 31), "dsm_ep_dispatch: bad shape");
  DSM_REQUIRE(n_tokens * std::min(topk, d->e_local) <= d->capacity || n_tokens == 0,
              "dsm_ep_dispatch: more rows per owner than the buffer's capacity");
  DSM_REQUIRE(counts && peer_base && done && epoch != 0, "dsm_ep_dispatch: NULL pointer or epoch 0");
  DSM_REQUIRE(n_tokens == 0 || (x && indices && perm && offsets && row_map), "dsm_ep_dispatch: NULL pointer");
  DSM_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0, "dsm_ep_dispatch: x must be 16-byte aligned");
  const int64_t pairs = n_tokens * topk;
  ep_dispatch_kernel<<<unsigned(std::min(pairs, kEpDispatchCtas) + 1), kEpCopyThreads, 0, as_stream(stream)>>>(
      geom_of(d), static_cast<const uint8_t*>(x), n_tokens, indices, perm, offsets, counts, pairs, topk, peer_base,
      row_map, done, epoch);
  return check_launch("ep_dispatch");
}

extern "C" int dsm_ep_receive(const dsm_ep_desc* d, const void* own_buffer, uint32_t epoch, int32_t* offsets,
                              int32_t* lperm, int32_t* n_valid, void* stream) {
  using namespace dsm;
  if (int rc = check_desc(d, "dsm_ep_receive")) return rc;
  DSM_REQUIRE(own_buffer && offsets && lperm && n_valid && epoch != 0, "dsm_ep_receive: NULL pointer or epoch 0");
  const size_t smem = (size_t(3) * d->world * d->e_local + d->e_local + 1) * 4;
  DSM_REQUIRE(smem <= 48 * 1024, "dsm_ep_receive: too many local experts");
  ep_receive_kernel<<<1, 1024, smem, as_stream(stream)>>>(geom_of(d), static_cast<const uint8_t*>(own_buffer), epoch,
                                                          offsets, lperm, n_valid);
  return check_launch("ep_receive");
}

extern "C" int dsm_ep_return(const dsm_ep_desc* d, const float* o_rows, const int32_t* n_valid,
                             const uint64_t* peer_base, uint32_t* done, uint32_t epoch, void* stream) {
  using namespace dsm;
  if (int rc = check_desc(d, "dsm_ep_return")) return rc;
  DSM_REQUIRE(o_rows && n_valid && peer_base && done && epoch != 0, "dsm_ep_return: NULL pointer or epoch 0");
  DSM_REQUIRE((int64_t(d->dim) * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(o_rows) & 15) == 0,
              "dsm_ep_return: rows must be 16-byte aligned");
  const int per = ep_return_per_sender(d->world);
  ep_return_kernel<<<unsigned(d->world * per), kEpCopyThreads, 0, as_stream(stream)>>>(geom_of(d), o_rows, n_valid,
                                                                                        peer_base, done, epoch, per);
  return check_launch("ep_return");
}

extern "C" int dsm_ep_wait_results(const dsm_ep_desc* d, const void* own_buffer, uint32_t epoch, void* stream) {
  using namespace dsm;
  if (int rc = check_desc(d, "dsm_ep_wait_results")) return rc;
  DSM_REQUIRE(own_buffer && epoch != 0, "dsm_ep_wait_results: NULL pointer or epoch 0");
  ep_wait_results_kernel<<<1, 32 * unsigned(ceil_div(d->world, 32)), 0, as_stream(stream)>>>(
      geom_of(d), static_cast<const uint8_t*>(own_buffer), epoch);
  return check_launch("ep_wait_results");
}

extern "C" int dsm_enable_peer_access(int peer_device) {
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return dsm::fail(DSM_ERR_CUDA, "dsm_enable_peer_access: cudaGetDevice");
  if (peer_device == cur) return DSM_OK;
  int can = 0;
  if (cudaDeviceCanAccessPeer(&can, cur, peer_device) != cudaSuccess || !can)
    return dsm::fail(DSM_ERR_UNSUPPORTED, "dsm_enable_peer_access: no peer access between these devices");
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();
    return DSM_OK;
  }
  if (e != cudaSuccess) return dsm::fail(DSM_ERR_CUDA, std::string("dsm_enable_peer_access: ") + cudaGetErrorString(e));
  return DSM_OK;
}

// ---- exchange buffers across processes (CUDA IPC) -------------------------------------------
namespace {
PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}
}  // namespace

extern "C" int dsm_ipc_get_handle(const void* ptr, void* handle, int64_t* offset) {
  using namespace dsm;
  DSM_REQUIRE(ptr && handle && offset, "dsm_ipc_get_handle: NULL pointer");
  auto range = address_range_fn();
  if (!range) return fail(DSM_ERR_CUDA, "dsm_ipc_get_handle: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(DSM_ERR_CUDA, "dsm_ipc_get_handle: not a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(DSM_ERR_CUDA, std::string("dsm_ipc_get_handle: ") + cudaGetErrorString(e));
  std::memcpy(handle, &h, sizeof(h));
  *offset = int64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return DSM_OK;
}

extern "C" int dsm_ipc_open(const void* handle, uint64_t* base) {
  using namespace dsm;
  DSM_REQUIRE(handle && base, "dsm_ipc_open: NULL pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(DSM_ERR_CUDA, std::string("dsm_ipc_open: ") + cudaGetErrorString(e));
  *base = reinterpret_cast<uint64_t>(p);
  return DSM_OK;
}

extern "C" int dsm_ipc_close(uint64_t base) {
  const cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return dsm::fail(DSM_ERR_CUDA, std::string("dsm_ipc_close: ") + cudaGetErrorString(e));
  return DSM_OK;
}
