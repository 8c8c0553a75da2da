// Grouped expert products at decode token counts: the routed experts' gather_mm /
// gather_qmm calls and the SwiGLU between them (dspark_mlx/model/moe.py:37-44, 132-149).
//
// Work unit = (expert e, 128-row tile of the output features, chunk of BN = 8*NT of the
// expert's staged rows). A persistent grid (one CTA per SM) walks the units; every CTA
// computes the unit list from the expert offsets itself, so no host round trip is needed.
//
// Per CTA: one producer warp issues, per pipeline stage (K chunk of 128), one bulk copy of
// the packed weight tile (two for the fused gate/up pair) and one of the BN staged
// activation rows into a ring of shared-memory stages (mbarrier complete_tx); eight
// consumer warps each own 16 weight rows, load their A fragments with one ld.shared.v4 per
// m16 tile (the packer stored them in fragment order), dequantise in registers (hardware
// e4m3 -> f16 conversion; f16 codes as they are), and run mma.sync m16n8k16 f16 x f16 ->
// fp32 against the activations. Weight streams are read with an L2 evict-first policy,
// activations with evict-last.
//
// Scales: the fp8 128x128 block scale is applied to each stage's fp32 partial sums; the
// per-expert multiplier from the packed header (f16 prescale) and the activation row scale
// are applied in the epilogue. fp4 and MLX affine experts are multiplied by the
// tensor-memory kernel (expert_tm.cu) at every token count.
//
// Epilogue of the gate/up kernel: g, u -> (optional bf16 rounding, as bf16 / affine
// weights give bf16 products in the reference) -> activation -> bf16 rounding (the
// reference casts h to x.dtype) -> staged f16 rows for the down kernel. Epilogue of the
// down kernel: fp32 rows of o (optionally rounded to bf16).
#include <algorithm>
#include <atomic>
#include <cmath>

#include "common.cuh"

namespace dsm {
namespace {

// Consumer warps share a 128-row tile as 8 m16 tiles; more warps give the in-register
// dequantisation (2 cvt + 1 multiply per 4 e2m1 codes) more issue slots.
constexpr int kConsumerWarps = 8;
constexpr int kMt = 8 / kConsumerWarps;  // m16 tiles per consumer warp
constexpr int kThreads = (kConsumerWarps + 1) * 32;

struct ExpertArgs {
  const uint8_t* wa;  // packed weights (gate or down)
  const uint8_t* wb;  // packed up weights (gate/up kernel) or nullptr
  const __half* xin;  // staged activation rows
  const float* act_scale;  // per staged row, or nullptr -> act_scale_const
  float act_scale_const;
  int64_t rows_cap;
  const int32_t* offsets;
  int n_experts;
  int out_rows;
  int rt_count;
  int kc_count;
  int group_size;
  int act;
  float limit;
  int round_gu;
  float h_scale;
  __half* h_out;
  int64_t h_rows_cap;
  float* o_out;
  const int32_t* o_row_map;  // down: staged row r is written to output row o_row_map[r] (NULL: r)
  int ldo;
  int round_o;
  int64_t n_rows;  // rows of the single group when offsets is NULL
  // single-matrix product only: K ranges per (row tile, row chunk), each writing an fp32
  // partial slab o_out + split * o_split_stride (rows [n_rows][ldo], staged-row order, no row
  // map); 0 or 1 = no split. k_per: 128-K chunks per range.
  int k_splits;
  int k_per;
  int64_t o_split_stride;
};

// rows [first, first + count) of group e (offsets == NULL: one group holding every row)
__device__ __forceinline__ int group_first(const ExpertArgs& a, int e) { return a.offsets ? a.offsets[e] : 0; }
__device__ __forceinline__ int group_count(const ExpertArgs& a, int e) {
  return a.offsets ? a.offsets[e + 1] - a.offsets[e] : int(a.n_rows);
}

// expert e owning unit u: the largest e with pre[e] <= u (pre[0] = 0, pre[E] = total)
__device__ __forceinline__ int find_expert(const int* pre, int n_experts, int u) {
  int lo = 0, hi = n_experts - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (pre[mid] <= u)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// SPLIT: the single-matrix product over K ranges (k_splits, k_per), each unit writing an fp32
// partial slab; a separate instance, so the unsplit kernels keep their code as it was.
template <int FMT, bool DUAL, int NT, bool SPLIT = false>
__global__ void __launch_bounds__(kThreads, 1) expert_kernel(const ExpertArgs a, int n_stages) {
  static_assert(!(SPLIT && DUAL), "K split: single-matrix products only");
  constexpr int BN = 8 * NT;
  constexpr int NM = DUAL ? 2 : 1;
  static_assert(FMT == DSM_WFMT_F16 || FMT == DSM_WFMT_FP8_B128, "f16 and fp8 tiles only");
  constexpr bool kBlockScaled = FMT == DSM_WFMT_FP8_B128;
  constexpr bool kTmp = kBlockScaled;
  extern __shared__ __align__(1024) uint8_t smem[];

  const int tile_b = tile_bytes(FMT, a.group_size);
  constexpr int act_b = BN * kStagePitch * 2;
  const int stage_b = NM * tile_b + act_b;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + int64_t(n_stages) * stage_b);
  uint64_t* empty = full + n_stages;
  int* pre = reinterpret_cast<int*>(empty + n_stages);
  volatile int* abort_flag = pre + a.n_experts + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.n_experts;
  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {  // units per expert, inclusive scan -> pre[1..E]
    int carry = 0;
    if (lane == 0) pre[0] = 0;
    for (int base = 0; base < E; base += 32) {
      const int e = base + lane;
      int v = 0;
      if (e < E) {
        const int cnt = group_count(a, e);
        v = cnt > 0 ? a.rt_count * ((cnt + BN - 1) / BN) * (SPLIT ? a.k_splits : 1) : 0;
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (e < E) pre[e + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  const int total = pre[E];
  const float* hdr_a = reinterpret_cast<const float*>(a.wa);
  const float* hdr_b = DUAL ? reinterpret_cast<const float*>(a.wb) : nullptr;
  const int64_t hdr_bytes = ceil_div(int64_t(E) * 4, kPackHeader) * kPackHeader;
  const uint8_t* tiles_a = a.wa + hdr_bytes;
  const uint8_t* tiles_b = DUAL ? a.wb + hdr_bytes : nullptr;

  if (warp == kConsumerWarps) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int e = find_expert(pre, E, u);
        const int cnt = group_count(a, e);
        const int nch = (cnt + BN - 1) / BN;
        const int local = u - pre[e];
        const int nsp = SPLIT ? a.k_splits : 1;
        const int rt = local / (nch * nsp), r2 = local % (nch * nsp);
        const int chunk = r2 % nch;
        const int kc0 = SPLIT ? (r2 / nch) * a.k_per : 0;
        const int kc1 = SPLIT ? min(a.kc_count, kc0 + a.k_per) : a.kc_count;
        const int64_t row0 = int64_t(group_first(a, e)) + int64_t(chunk) * BN;
        const int64_t tile0 = (int64_t(e) * a.rt_count + rt) * a.kc_count;
        for (int kc = kc0; kc < kc1; ++kc) {
          if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* st = smem + int64_t(s) * stage_b;
          mbar_arrive_expect_tx(&full[s], uint32_t(stage_b));
          bulk_g2s(st, tiles_a + (tile0 + kc) * tile_b, uint32_t(tile_b), &full[s], pol_w);
          if (DUAL) bulk_g2s(st + tile_b, tiles_b + (tile0 + kc) * tile_b, uint32_t(tile_b), &full[s], pol_w);
          bulk_g2s(st + NM * tile_b, a.xin + (int64_t(kc) * a.rows_cap + row0) * kStagePitch, uint32_t(act_b),
                   &full[s], pol_x);
          if (++s == n_stages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // let copies already in flight land before the CTA retires (bounded: ~100 us)
        for (int i = 0; i < 100; ++i) __nanosleep(1000);
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int g = lane >> 2, q = lane & 3;
  int s = 0;
  uint32_t ph = 0;
  for (int u = blockIdx.x; u < total; u += gridDim.x) {
    const int e = find_expert(pre, E, u);
    const int off = group_first(a, e);
    const int cnt = group_count(a, e);
    const int nch = (cnt + BN - 1) / BN;
    const int local = u - pre[e];
    const int nsp = SPLIT ? a.k_splits : 1;
    const int rt = local / (nch * nsp), r2 = local % (nch * nsp);
    const int chunk = r2 % nch, ks = r2 / nch;
    const int kc0 = SPLIT ? ks * a.k_per : 0;
    const int kc1 = SPLIT ? min(a.kc_count, kc0 + a.k_per) : a.kc_count;

    float acc[NM][kMt][NT][4];
    float tmp[kTmp ? NM : 1][kMt][NT][4];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
      for (int i = 0; i < kMt; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            acc[m][i][j][c] = 0.f;
            if (kTmp) tmp[m < (kTmp ? NM : 1) ? m : 0][i][j][c] = 0.f;
          }

    bool ok = true;
    for (int kc = kc0; kc < kc1; ++kc) {
      if (*abort_flag || !mbar_wait(&full[s], ph)) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      const uint32_t st = smem_u32(smem + int64_t(s) * stage_b);
      const uint32_t sx = st + NM * tile_b;
      // ---- per-format stage compute
      if constexpr (FMT == DSM_WFMT_F16) {
#pragma unroll
        for (int sl = 0; sl < 8; ++sl) {
          uint32_t A[NM][kMt][4];
#pragma unroll
          for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int i = 0; i < kMt; ++i) {
              const uint4 v = lds128(st + m * tile_b + ((sl * 8 + kMt * warp + i) * 32 + lane) * 16);
              A[m][i][0] = v.x;
              A[m][i][1] = v.z;
              A[m][i][2] = v.y;
              A[m][i][3] = v.w;
            }
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const uint2 xb = lds64(sx + (j * 8 + g) * (kStagePitch * 2) + sl * 32 + q * 8);
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
              for (int i = 0; i < kMt; ++i) mma_f16(acc[m][i][j], A[m][i], xb.x, xb.y);
          }
        }
      } else {  // FP8_B128: 128x128 block scale applied to the stage's fp32 partials
#pragma unroll
        for (int sl = 0; sl < 4; ++sl) {
          uint32_t A[NM][kMt][2][4];  // [matrix][m16 tile][mma 0/1][regs]
#pragma unroll
          for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int i = 0; i < kMt; ++i) {
              const uint4 v = lds128(st + m * tile_b + ((sl * 8 + kMt * warp + i) * 32 + lane) * 16);
              e4m3x4_to_f16(v.x, A[m][i][0][0], A[m][i][0][2]);
              e4m3x4_to_f16(v.y, A[m][i][1][0], A[m][i][1][2]);
              e4m3x4_to_f16(v.z, A[m][i][0][1], A[m][i][0][3]);
              e4m3x4_to_f16(v.w, A[m][i][1][1], A[m][i][1][3]);
            }
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const uint4 xb = lds128(sx + (j * 8 + g) * (kStagePitch * 2) + sl * 64 + q * 16);
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
              for (int i = 0; i < kMt; ++i) {
                mma_f16(tmp[m][i][j], A[m][i][0], xb.x, xb.y);
                mma_f16(tmp[m][i][j], A[m][i][1], xb.z, xb.w);
              }
          }
        }
        if constexpr (kBlockScaled) {
#pragma unroll
          for (int m = 0; m < NM; ++m) {
            const float sc = __uint_as_float(lds32(st + m * tile_b + tile_code_bytes(FMT)));
#pragma unroll
            for (int i = 0; i < kMt; ++i)
#pragma unroll
              for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  acc[m][i][j][c] = fmaf(sc, tmp[m][i][j][c], acc[m][i][j][c]);
                  tmp[m][i][j][c] = 0.f;
                }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == n_stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    if (!ok) break;

    // ---------------------------------------------------------------- epilogue
    const float wmul_a = hdr_a[e];
    const float wmul_b = DUAL ? hdr_b[e] : 1.f;
#pragma unroll
    for (int i = 0; i < kMt; ++i)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int col = chunk * BN + j * 8 + 2 * q + (c & 1);
          if (col >= cnt) continue;
          const int rloc = 16 * (kMt * warp + i) + g + ((c & 2) ? 8 : 0);
          const int64_t r = int64_t(off) + col;
          const float xs = a.act_scale ? a.act_scale[r] : a.act_scale_const;
          if constexpr (DUAL) {
            float gv = acc[0][i][j][c] * xs * wmul_a;
            float uv = acc[DUAL ? 1 : 0][i][j][c] * xs * wmul_b;
            if (a.round_gu & 1) {
              gv = bf16_round(gv);
              uv = bf16_round(uv);
            }
            float h = swiglu(gv, uv, a.act, a.limit);
            if (a.round_gu & 2) h = bf16_round(h);
            a.h_out[(int64_t(rt) * a.h_rows_cap + r) * kStagePitch + rloc] = __float2half_rn(h * a.h_scale);
          } else {
            const int d = rt * kTileRows + rloc;
            if (d >= a.out_rows) continue;
            float v = acc[0][i][j][c] * xs * wmul_a;
            if constexpr (SPLIT) {  // a partial of the K range: summed and rounded by the split sum
              a.o_out[int64_t(ks) * a.o_split_stride + r * a.ldo + d] = v;
              continue;
            }
            if (a.round_o) v = bf16_round(v);
            const int64_t orow = a.o_row_map ? int64_t(a.o_row_map[r]) : r;
            a.o_out[orow * a.ldo + d] = v;
          }
        }
  }
}

template <int FMT, bool DUAL, int NT, bool SPLIT = false>
int launch_expert(const ExpertArgs& a, cudaStream_t stream) {
  const int tile_b = tile_bytes(FMT, a.group_size);
  const int act_b = 8 * NT * kStagePitch * 2;
  const int stage_b = (DUAL ? 2 : 1) * tile_b + act_b;
  const int budget = 200 * 1024;
  int n_stages = std::min(8, budget / stage_b);
  if (n_stages < 2) return fail(DSM_ERR_UNSUPPORTED, "expert kernel: tile too large for the shared-memory ring");
  const size_t smem = size_t(n_stages) * stage_b + size_t(2 * n_stages) * 8 + size_t(a.n_experts + 2) * 4;
  auto kern = expert_kernel<FMT, DUAL, NT, SPLIT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return check_launch("expert kernel smem attribute");
  kern<<<persistent_ctas(), kThreads, smem, stream>>>(a, n_stages);
  return check_launch("expert kernel");
}

template <bool DUAL>
int dispatch(int wfmt, int nt, const ExpertArgs& a, cudaStream_t s) {
#define DSM_NT_CASES(F)                                    \
  if (nt == 1) return launch_expert<F, DUAL, 1>(a, s);     \
  if (nt == 2) return launch_expert<F, DUAL, 2>(a, s);     \
  return launch_expert<F, DUAL, 4>(a, s);
  switch (wfmt) {
    case DSM_WFMT_F16: { DSM_NT_CASES(DSM_WFMT_F16) }
    case DSM_WFMT_FP8_B128: { DSM_NT_CASES(DSM_WFMT_FP8_B128) }
    default: return fail(DSM_ERR_INVALID_ARGUMENT, "expert kernel: unknown weight format");
  }
#undef DSM_NT_CASES
}

// the K-split instances: single matrix, up to eight n8 tiles (a group's rows whole)
int dispatch_split(int wfmt, int nt, const ExpertArgs& a, cudaStream_t s) {
#define DSM_NT_CASES(F)                                          \
  if (nt == 1) return launch_expert<F, false, 1, true>(a, s);    \
  if (nt == 2) return launch_expert<F, false, 2, true>(a, s);    \
  if (nt == 4) return launch_expert<F, false, 4, true>(a, s);    \
  return launch_expert<F, false, 8, true>(a, s);
  switch (wfmt) {
    case DSM_WFMT_F16: { DSM_NT_CASES(DSM_WFMT_F16) }
    case DSM_WFMT_FP8_B128: { DSM_NT_CASES(DSM_WFMT_FP8_B128) }
    default: return fail(DSM_ERR_INVALID_ARGUMENT, "expert kernel: unknown weight format");
  }
#undef DSM_NT_CASES
}

// n-tile count from the average rows per expert: decode draft blocks put one or two rows
// on most experts, so one n8 tile keeps the tensor-core work per weight byte minimal. A
// wider tile re-reads each weight tile less often, but only while the grid stays full:
// with few busy experts (the shared expert is one group holding every token) narrower
// tiles give more work units, and the re-reads of a tile are served from L2. The grid is
// this launch's persistent grid: a slice of the SMs when the shared expert runs beside the
// routed products, where wider tiles (fewer re-reads per SM) win. Four n8 tiles at most:
// eight-tile units are bound by their mma.sync work per weight byte (a 56-row LM head ran
// 0.344 ms in 32-row units, 0.311 ms in 64-row units and 0.231 ms on the tcgen05 kernel), so
// single matrices above 32 rows take the tcgen05 kernel (dsm_linear), and eight-tile units
// serve only the K-split products when the tcgen05 kernel is switched off.
int pick_nt(int64_t n_rows, int n_experts, int rt_count) {
  const int64_t busy = std::max<int64_t>(1, std::min<int64_t>(n_rows, n_experts));
  const double avg = double(n_rows) / double(busy);
  int nt = avg <= 8.0 ? 1 : (avg <= 16.0 ? 2 : 4);
  while (nt > 1) {
    const int64_t units = busy * int64_t(std::ceil(avg / (8.0 * nt))) * rt_count;
    if (units >= 2 * int64_t(persistent_ctas())) break;
    nt >>= 1;
  }
  return nt;
}

// per host thread: a caller's choice never changes another thread's launches
thread_local int g_regime = 0;

// The tcgen05 kernel pays off once an expert's weight tile is reused by many rows: with
// 128-row MMA tiles, from about 64 rows per busy expert on average.
// min_rows: rows per busy expert from which the tcgen05 kernel runs. A single matrix with
// many row tiles (dsm_linear: an LM head, a wide projection) switches above 32 rows: there
// the streaming kernel needs its eight-tile units, whose mma.sync work per weight byte is
// the bound (measured on a 129,280 x 4096 bf16 LM head: 32 rows streaming 182 us, 56 rows
// streaming 315 us, 64 rows on tcgen05 235 us).
bool use_tc(int wfmt, int64_t n_rows, int n_experts, int min_rows = 64) {
  if (!tc_supports(wfmt)) return false;
  const int r = g_regime;
  if (r == 1) return false;
  if (r == 2) return true;
  const int64_t busy = std::max<int64_t>(1, std::min<int64_t>(n_rows, n_experts));
  return n_rows >= int64_t(min_rows) * busy;
}

int check_common(int wfmt, int group_size, const int32_t* offsets, int n_experts) {
  DSM_REQUIRE(wfmt >= DSM_WFMT_F16 && wfmt <= DSM_WFMT_AFFINE4, "expert: unknown weight format");
  DSM_REQUIRE(n_experts >= 1 && n_experts <= 4096, "expert: n_experts out of range");
  DSM_REQUIRE(offsets != nullptr || n_experts == 1, "expert: offsets may be NULL only for a single group");
  if (wfmt == DSM_WFMT_AFFINE8)
    DSM_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, "expert: affine8 group_size 32/64/128");
  if (wfmt == DSM_WFMT_AFFINE4) DSM_REQUIRE(group_size == 64 || group_size == 128, "expert: affine4 group_size 64/128");
  return DSM_OK;
}

}  // namespace
}  // namespace dsm

extern "C" int dsm_expert_gate_up(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int dim,
                                  const int32_t* offsets, int n_experts, int wfmt, int group_size,
                                  const void* w1_packed, const void* w3_packed, int inter, int act,
                                  float swiglu_limit, int round_gu, void* h_staged, float h_scale, int64_t n_rows,
                                  void* stream) {
  using namespace dsm;
  if (int rc = check_common(wfmt, group_size, offsets, n_experts)) return rc;
  DSM_REQUIRE(dim > 0 && inter > 0 && n_rows >= 0, "dsm_expert_gate_up: bad shape");
  DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(n_rows), "dsm_expert_gate_up: rows_cap too small");
  DSM_REQUIRE(act == DSM_ACT_SWIGLU_CLAMP || act == DSM_ACT_SILU_MUL_BF16, "dsm_expert_gate_up: bad act");
  DSM_REQUIRE(x_staged && x_row_scale && w1_packed && w3_packed && h_staged, "dsm_expert_gate_up: NULL pointer");
  if (n_rows == 0) return DSM_OK;
  ExpertArgs a{};
  a.wa = static_cast<const uint8_t*>(w1_packed);
  a.wb = static_cast<const uint8_t*>(w3_packed);
  a.xin = static_cast<const __half*>(x_staged);
  a.act_scale = x_row_scale;
  a.act_scale_const = 1.f;
  a.rows_cap = rows_cap;
  a.offsets = offsets;
  a.n_rows = n_rows;
  a.n_experts = n_experts;
  a.out_rows = inter;
  a.rt_count = int(ceil_div(inter, kTileRows));
  a.kc_count = int(ceil_div(dim, kChunkK));
  a.group_size = group_size > 0 ? group_size : 64;
  a.act = act;
  a.limit = swiglu_limit;
  a.round_gu = round_gu;
  a.h_scale = h_scale;
  a.h_out = static_cast<__half*>(h_staged);
  a.h_rows_cap = rows_cap;
  if (tm_supports(wfmt))
    return expert_tm_gate_up(wfmt, group_size, x_staged, x_row_scale, rows_cap, dim, offsets, n_experts, w1_packed,
                             w3_packed, inter, act, swiglu_limit, round_gu, h_staged, h_scale, n_rows, stream);
  if (use_tc(wfmt, n_rows, n_experts))
    return expert_tc_gate_up(wfmt, x_staged, x_row_scale, rows_cap, dim, offsets, n_experts, w1_packed, w3_packed, inter,
                             act, swiglu_limit, round_gu, h_staged, h_scale, n_rows, stream);
  return dispatch<true>(wfmt, pick_nt(n_rows, n_experts, a.rt_count), a, as_stream(stream));
}

extern "C" int dsm_expert_down(const void* h_staged, float h_scale, int64_t rows_cap, int inter,
                               const int32_t* offsets, int n_experts, int wfmt, int group_size, const void* w2_packed,
                               int dim, int round_o, float* o_rows, int ldo, const int32_t* o_row_map,
                               int64_t n_rows, void* stream) {
  using namespace dsm;
  if (int rc = check_common(wfmt, group_size, offsets, n_experts)) return rc;
  DSM_REQUIRE(dim > 0 && inter > 0 && n_rows >= 0 && ldo >= dim, "dsm_expert_down: bad shape");
  DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(n_rows), "dsm_expert_down: rows_cap too small");
  DSM_REQUIRE(h_scale > 0.f, "dsm_expert_down: h_scale must be positive");
  DSM_REQUIRE(h_staged && w2_packed && o_rows, "dsm_expert_down: NULL pointer");
  if (n_rows == 0) return DSM_OK;
  ExpertArgs a{};
  a.wa = static_cast<const uint8_t*>(w2_packed);
  a.wb = nullptr;
  a.xin = static_cast<const __half*>(h_staged);
  a.act_scale = nullptr;
  a.act_scale_const = 1.f / h_scale;
  a.rows_cap = rows_cap;
  a.offsets = offsets;
  a.n_rows = n_rows;
  a.n_experts = n_experts;
  a.out_rows = dim;
  a.rt_count = int(ceil_div(dim, kTileRows));
  a.kc_count = int(ceil_div(inter, kChunkK));
  a.group_size = group_size > 0 ? group_size : 64;
  a.o_out = o_rows;
  a.o_row_map = o_row_map;
  a.ldo = ldo;
  a.round_o = round_o;
  if (tm_supports(wfmt))
    return expert_tm_down(wfmt, group_size, h_staged, h_scale, rows_cap, inter, offsets, n_experts, w2_packed, dim,
                          round_o, o_rows, ldo, o_row_map, n_rows, stream);
  if (use_tc(wfmt, n_rows, n_experts))
    return expert_tc_down(wfmt, h_staged, h_scale, rows_cap, inter, offsets, n_experts, w2_packed, dim, round_o, o_rows, ldo,
                          o_row_map, n_rows, stream);
  return dispatch<false>(wfmt, pick_nt(n_rows, n_experts, a.rt_count), a, as_stream(stream));
}

extern "C" int dsm_linear(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim, int wfmt,
                          int group_size, const void* w_packed, int out_dim, float* o_rows, int ldo, int64_t n_rows,
                          void* stream) {
  using namespace dsm;
  if (int rc = check_common(wfmt, group_size, nullptr, 1)) return rc;
  DSM_REQUIRE(out_dim > 0 && k_dim > 0 && n_rows >= 0 && ldo >= out_dim, "dsm_linear: bad shape");
  DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(n_rows), "dsm_linear: rows_cap too small");
  DSM_REQUIRE(x_staged && x_row_scale && w_packed && o_rows, "dsm_linear: NULL pointer");
  if (n_rows == 0) return DSM_OK;
  if (tm_supports(wfmt))
    return expert_tm_down(wfmt, group_size, x_staged, 1.f, rows_cap, k_dim, nullptr, 1, w_packed, out_dim, 0, o_rows,
                          ldo, nullptr, n_rows, stream, x_row_scale);
  if (use_tc(wfmt, n_rows, 1, 33))
    return expert_tc_down(wfmt, x_staged, 1.f, rows_cap, k_dim, nullptr, 1, w_packed, out_dim, 0, o_rows, ldo, nullptr,
                          n_rows, stream, x_row_scale);
  ExpertArgs a{};
  a.wa = static_cast<const uint8_t*>(w_packed);
  a.wb = nullptr;
  a.xin = static_cast<const __half*>(x_staged);
  a.act_scale = x_row_scale;
  a.act_scale_const = 1.f;
  a.rows_cap = rows_cap;
  a.offsets = nullptr;
  a.n_rows = n_rows;
  a.n_experts = 1;
  a.out_rows = out_dim;
  a.rt_count = int(ceil_div(out_dim, kTileRows));
  a.kc_count = int(ceil_div(k_dim, kChunkK));
  a.group_size = group_size > 0 ? group_size : 64;
  a.o_out = o_rows;
  a.o_row_map = nullptr;
  a.ldo = ldo;
  a.round_o = 0;
  return dispatch<false>(wfmt, pick_nt(n_rows, 1, a.rt_count), a, as_stream(stream));
}

extern "C" int dsm_grouped_linear(const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim,
                                  int wfmt, int group_size, const void* w_packed, int n_groups,
                                  const int32_t* offsets, int out_dim, float* o_rows, int ldo,
                                  const int32_t* o_row_map, int64_t n_rows, void* stream) {
  using namespace dsm;
  if (int rc = check_common(wfmt, group_size, offsets, n_groups)) return rc;
  DSM_REQUIRE(out_dim > 0 && k_dim > 0 && n_rows >= 0 && ldo >= out_dim, "dsm_grouped_linear: bad shape");
  DSM_REQUIRE(rows_cap >= dsm_stage_rows_cap(n_rows), "dsm_grouped_linear: rows_cap too small");
  DSM_REQUIRE(x_staged && x_row_scale && w_packed && o_rows, "dsm_grouped_linear: NULL pointer");
  if (n_rows == 0) return DSM_OK;
  if (tm_supports(wfmt))
    return expert_tm_down(wfmt, group_size, x_staged, 1.f, rows_cap, k_dim, offsets, n_groups, w_packed, out_dim, 0,
                          o_rows, ldo, o_row_map, n_rows, stream, x_row_scale);
  if (use_tc(wfmt, n_rows, n_groups))
    return expert_tc_down(wfmt, x_staged, 1.f, rows_cap, k_dim, offsets, n_groups, w_packed, out_dim, 0, o_rows, ldo,
                          o_row_map, n_rows, stream, x_row_scale);
  ExpertArgs a{};
  a.wa = static_cast<const uint8_t*>(w_packed);
  a.wb = nullptr;
  a.xin = static_cast<const __half*>(x_staged);
  a.act_scale = x_row_scale;
  a.act_scale_const = 1.f;
  a.rows_cap = rows_cap;
  a.offsets = offsets;
  a.n_rows = n_rows;
  a.n_experts = n_groups;
  a.out_rows = out_dim;
  a.rt_count = int(ceil_div(out_dim, kTileRows));
  a.kc_count = int(ceil_div(k_dim, kChunkK));
  a.group_size = group_size > 0 ? group_size : 64;
  a.o_out = o_rows;
  a.o_row_map = o_row_map;
  a.ldo = ldo;
  a.round_o = 0;
  return dispatch<false>(wfmt, pick_nt(n_rows, n_groups, a.rt_count), a, as_stream(stream));
}

namespace dsm {
int expert_regime() { return g_regime; }

int expert_stream_split(int wfmt, int group_size, const void* x_staged, const float* x_row_scale, int64_t rows_cap,
                        int k_dim, const int32_t* offsets, int n_groups, const void* w_packed, int out_dim,
                        int64_t n_rows, int max_splits, float* parts, void* stream, int* splits_used) {
  *splits_used = 1;
  if ((wfmt != DSM_WFMT_F16 && wfmt != DSM_WFMT_FP8_B128) || n_rows <= 0) return DSM_OK;
  const int rt = int(ceil_div(out_dim, kTileRows)), kcs = int(ceil_div(k_dim, kChunkK));
  const int64_t busy = std::max<int64_t>(1, std::min<int64_t>(n_rows, n_groups));
  const double avg = double(n_rows) / double(busy);
  // Above 32 rows per group the tcgen05 kernel takes the ranges (units of up to 256 rows);
  // below, the streaming kernel in the narrowest unit holding a group's rows. Either way each
  // weight tile is streamed once per K range, and the K ranges, not row chunks, fill the SMs.
  const bool tc = use_tc(wfmt, n_rows, n_groups, 33);
  const int nt = avg <= 8.0 ? 1 : (avg <= 16.0 ? 2 : (avg <= 32.0 ? 4 : 8));
  const double unit_rows = tc ? 256.0 : 8.0 * nt;
  const int64_t units = busy * int64_t(std::ceil(avg / unit_rows)) * rt;
  int splits = int(std::min<int64_t>({int64_t(max_splits), int64_t(kcs), int64_t(persistent_ctas()) / units}));
  if (splits <= 1) return DSM_OK;
  const int k_per = int(ceil_div(kcs, splits));
  splits = int(ceil_div(kcs, k_per));  // no empty range
  if (splits <= 1) return DSM_OK;
  if (tc) {
    const int rc = expert_tc_split(wfmt, x_staged, x_row_scale, rows_cap, k_dim, offsets, n_groups, w_packed, out_dim,
                                   n_rows, splits, k_per, parts, stream);
    if (rc == DSM_OK) *splits_used = splits;
    return rc;
  }
  ExpertArgs a{};
  a.wa = static_cast<const uint8_t*>(w_packed);
  a.wb = nullptr;
  a.xin = static_cast<const __half*>(x_staged);
  a.act_scale = x_row_scale;
  a.act_scale_const = 1.f;
  a.rows_cap = rows_cap;
  a.offsets = offsets;
  a.n_rows = n_rows;
  a.n_experts = n_groups;
  a.out_rows = out_dim;
  a.rt_count = rt;
  a.kc_count = kcs;
  a.group_size = group_size > 0 ? group_size : 64;
  a.o_out = parts;
  a.o_row_map = nullptr;
  a.ldo = out_dim;
  a.round_o = 0;
  a.k_splits = splits;
  a.k_per = k_per;
  a.o_split_stride = n_rows * int64_t(out_dim);
  const int rc = dispatch_split(wfmt, nt, a, as_stream(stream));
  if (rc == DSM_OK) *splits_used = splits;
  return rc;
}
}  // namespace dsm

extern "C" int dsm_set_expert_regime(int regime) {
  DSM_REQUIRE(regime >= 0 && regime <= 2, "dsm_set_expert_regime: regime must be 0, 1 or 2");
  dsm::g_regime = regime;
  return DSM_OK;
}
