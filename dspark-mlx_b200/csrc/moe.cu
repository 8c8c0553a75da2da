// dsm_moe_forward: the whole MoE.__call__ (dspark_mlx/model/moe.py:151-161) in one call:
// router -> permutation -> staged activations -> fused gate/up + activation -> down ->
// (shared expert: same kernels, one group holding every token) -> weighted combine.
// All scratch comes from the caller's workspace, carved up below.
//
// The shared expert runs next to the routed products: its kernels go to a side stream
// (forked from the caller's stream after staging, joined before the combine) on a small
// slice of the SMs, and the routed kernels' persistent grids leave that slice free. The
// routed products are HBM-bound and keep their bandwidth on the remaining SMs, while the
// shared expert (one dense matrix, few rows) is bound by latency rather than bandwidth and
// would otherwise add its whole duration to the step. Only decode-sized calls overlap: with
// thousands of tokens both products are compute-bound, and splitting the SMs between them
// gains nothing.
#include "common.cuh"

namespace dsm {
namespace {

struct Carve {
  uint8_t* base;
  size_t used = 0;
  void* take(size_t bytes) {
    void* p = base ? base + used : nullptr;
    used += (bytes + 255) & ~size_t(255);
    return p;
  }
};

// Per thread and device: the side stream and fork/join events, created on first use and
// kept for the life of the thread (the library allocates no device memory for them).
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  bool ready = false;
};

SideStream* side_stream() {
  thread_local SideStream per_device[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  SideStream& ss = per_device[dev];
  if (!ss.ready) {
    if (cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    if (cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess)
      return nullptr;
    ss.ready = true;
  }
  return &ss;
}

constexpr int kSharedCtas = 16;        // SMs given to the shared expert while the routed products run
constexpr int64_t kOverlapTokens = 2048;  // largest call that overlaps the shared expert

struct Layout {
  void* scores;
  float* weights;
  int32_t* indices;
  int32_t *counts, *offsets, *perm, *inv;
  void* perm_ws;
  size_t perm_ws_bytes;
  void *xs_r, *hs_r;
  float* xscale_r;
  float* o_r;
  int32_t* off_s;
  void *xs_s, *hs_s;
  float* xscale_s;
  float* o_s;
  int64_t cap_r, cap_s;
};

size_t carve(const dsm_moe_desc* d, void* ws, Layout* L, bool own_routing) {
  Carve c{static_cast<uint8_t*>(ws)};
  const int64_t N = d->n_tokens, P = N * d->topk;
  L->cap_r = dsm_stage_rows_cap(P);
  L->cap_s = dsm_stage_rows_cap(N);
  L->scores = c.take(dsm_router_workspace_bytes(N, d->dim, d->n_experts));
  if (own_routing) {
    L->weights = static_cast<float*>(c.take(size_t(P) * 4));
    L->indices = static_cast<int32_t*>(c.take(size_t(P) * 4));
  }
  L->counts = static_cast<int32_t*>(c.take(size_t(d->n_experts) * 4));
  L->offsets = static_cast<int32_t*>(c.take(size_t(d->n_experts + 1) * 4));
  L->perm = static_cast<int32_t*>(c.take(size_t(P) * 4));
  L->inv = static_cast<int32_t*>(c.take(size_t(P) * 4));
  L->perm_ws_bytes = dsm_permute_workspace_bytes(P, d->n_experts);
  L->perm_ws = c.take(L->perm_ws_bytes);
  L->xs_r = c.take(dsm_stage_bytes(L->cap_r, d->dim));
  L->xscale_r = static_cast<float*>(c.take(size_t(L->cap_r) * 4));
  L->hs_r = c.take(dsm_stage_bytes(L->cap_r, d->inter));
  L->o_r = static_cast<float*>(c.take(size_t(P) * d->dim * 4));
  if (d->s1) {
    L->off_s = static_cast<int32_t*>(c.take(16));
    L->xs_s = c.take(dsm_stage_bytes(L->cap_s, d->dim));
    L->xscale_s = static_cast<float*>(c.take(size_t(L->cap_s) * 4));
    L->hs_s = c.take(dsm_stage_bytes(L->cap_s, d->shared_inter));
    L->o_s = static_cast<float*>(c.take(size_t(N) * d->dim * 4));
  } else {
    L->off_s = nullptr;
    L->xs_s = L->hs_s = nullptr;
    L->xscale_s = L->o_s = nullptr;
  }
  return c.used;
}

}  // namespace
}  // namespace dsm

extern "C" size_t dsm_moe_workspace_bytes(const dsm_moe_desc* d) {
  if (!d) return 0;
  dsm::Layout L;
  return dsm::carve(d, nullptr, &L, true);
}

extern "C" int dsm_moe_forward(const dsm_moe_desc* d, const void* x, int x_dtype, const void* input_ids, int ids_dtype,
                               int64_t n_ids, void* y, float* route_weights_out, int32_t* route_indices_out,
                               void* workspace, size_t workspace_bytes, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(d != nullptr, "dsm_moe_forward: desc is NULL");
  DSM_REQUIRE(d->n_tokens >= 0 && d->dim > 0 && d->inter > 0 && d->n_experts > 0 && d->topk > 0,
              "dsm_moe_forward: bad shape");
  DSM_REQUIRE(!d->s1 || (d->s2 && d->s3 && d->shared_inter > 0), "dsm_moe_forward: incomplete shared expert");
  if (d->n_tokens == 0) return DSM_OK;
  DSM_REQUIRE(x && y && workspace, "dsm_moe_forward: NULL pointer");
  if (workspace_bytes < dsm_moe_workspace_bytes(d)) return fail(DSM_ERR_WORKSPACE, "dsm_moe_forward: workspace too small");
  Layout L;
  carve(d, workspace, &L, true);
  if (route_weights_out) L.weights = route_weights_out;
  if (route_indices_out) L.indices = route_indices_out;
  const int64_t N = d->n_tokens, P = N * d->topk;
  int rc = dsm_router(x, x_dtype, N, d->dim, d->gate_weight, d->n_experts, d->tid2eid ? nullptr : d->gate_bias,
                      d->tid2eid, d->vocab, input_ids, ids_dtype, n_ids, d->topk, d->score_func, d->route_scale,
                      L.scores, L.weights, L.indices, stream);
  if (rc) return rc;
  rc = dsm_permute(L.indices, P, d->n_experts, L.counts, L.offsets, L.perm, L.inv, L.perm_ws, L.perm_ws_bytes, stream);
  if (rc) return rc;
  // routed rows (expert order) and, for the shared expert, every token in order: one launch
  rc = stage_rows_pair(x, x_dtype, N, d->dim, L.perm, P, d->topk, L.xs_r, L.cap_r, L.xscale_r, d->s1 ? N : 0, L.xs_s,
                       L.cap_s, L.xscale_s, stream);
  if (rc) return rc;
  const float hs = h_scale_for(d->act, d->swiglu_limit);
  auto routed = [&]() -> int {
    int r = dsm_expert_gate_up(L.xs_r, L.xscale_r, L.cap_r, d->dim, L.offsets, d->n_experts, d->wfmt, d->group_size,
                               d->w1, d->w3, d->inter, d->act, d->swiglu_limit, d->round_gu, L.hs_r, hs, P, stream);
    if (r) return r;
    return dsm_expert_down(L.hs_r, hs, L.cap_r, d->inter, L.offsets, d->n_experts, d->wfmt, d->group_size, d->w2,
                           d->dim, d->round_o, L.o_r, d->dim, nullptr, P, stream);
  };
  auto shared = [&](void* st) -> int {
    int r = dsm_expert_gate_up(L.xs_s, L.xscale_s, L.cap_s, d->dim, nullptr, 1, d->shared_wfmt, d->shared_group_size,
                               d->s1, d->s3, d->shared_inter, d->act, d->swiglu_limit, d->shared_round_gu, L.hs_s,
                               hs, N, st);
    if (r) return r;
    return dsm_expert_down(L.hs_s, hs, L.cap_s, d->shared_inter, nullptr, 1, d->shared_wfmt, d->shared_group_size,
                           d->s2, d->dim, d->shared_round_o, L.o_s, d->dim, nullptr, N, st);
  };
  SideStream* side = d->s1 && N <= kOverlapTokens && num_sms() >= 4 * kSharedCtas ? side_stream() : nullptr;
  if (side) {
    cudaStream_t main = as_stream(stream);
    if (cudaEventRecord(side->fork, main) != cudaSuccess || cudaStreamWaitEvent(side->s, side->fork, 0) != cudaSuccess)
      return check_launch("dsm_moe_forward: fork");
    {
      GridLimit g(kSharedCtas);
      if ((rc = shared(side->s))) return rc;
    }
    if (cudaEventRecord(side->join, side->s) != cudaSuccess) return check_launch("dsm_moe_forward: join record");
    {
      GridLimit g(num_sms() - kSharedCtas);
      if ((rc = routed())) return rc;
    }
    if (cudaStreamWaitEvent(main, side->join, 0) != cudaSuccess) return check_launch("dsm_moe_forward: join");
  } else {
    if ((rc = routed())) return rc;
    if (d->s1 && (rc = shared(stream))) return rc;
  }
  const int y_dtype = x_dtype;
  return dsm_combine(L.o_r, L.inv, L.weights, N, d->topk, d->dim, L.o_s, y, y_dtype, stream);
}
