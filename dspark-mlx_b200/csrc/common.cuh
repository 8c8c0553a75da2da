// Shared device/host helpers of libdsm (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <type_traits>

#include "dsm.h"

namespace dsm {

// ------------------------------------------------------------------------------------------
// host-side status plumbing
// ------------------------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_launch(const char* what);

#define DSM_REQUIRE(cond, msg)                                   \
  do {                                                           \
    if (!(cond)) return ::dsm::fail(DSM_ERR_INVALID_ARGUMENT, msg); \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
int num_sms();
// CTAs of a persistent expert kernel launched by this thread: every SM, unless a GridLimit
// in scope narrows it (two such kernels then share the GPU on disjoint SMs)
int persistent_ctas();
struct GridLimit {
  explicit GridLimit(int ctas);
  ~GridLimit();
  GridLimit(const GridLimit&) = delete;
  GridLimit& operator=(const GridLimit&) = delete;

 private:
  int prev_;
};

// tcgen05 grouped products at large token counts (expert_tc.cu): fp8 block-scaled and f16
bool tc_supports(int wfmt);
int expert_tc_gate_up(int wfmt, const void* x_staged, const float* x_row_scale, int64_t rows_cap, int dim,
                      const int32_t* offsets, int n_experts, const void* w1, const void* w3, int inter, int act,
                      float limit, int round_gu, void* h_staged, float h_scale, int64_t n_rows, void* stream);
// x_row_scale (optional): per-row activation scales instead of the constant 1 / h_scale
// (a plain linear layer over rows staged by dsm_stage_rows)
int expert_tc_down(int wfmt, const void* h_staged, float h_scale, int64_t rows_cap, int inter, const int32_t* offsets,
                   int n_experts, const void* w2, int dim, int round_o, float* o_rows, int ldo,
                   const int32_t* o_row_map, int64_t n_rows, void* stream, const float* x_row_scale = nullptr);
// the single-matrix (grouped) product with K split into k_splits ranges of k_per 128-K chunks,
// fp32 partial slabs parts[split][n_rows][out_dim] in staged-row order
int expert_tc_split(int wfmt, const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim,
                    const int32_t* offsets, int n_groups, const void* w_packed, int out_dim, int64_t n_rows,
                    int k_splits, int k_per, float* parts, void* stream);
// fp4 and affine experts at every token count (expert_tm.cu): weights dequantised into
// tensor memory
bool tm_supports(int wfmt);
int expert_tm_gate_up(int wfmt, int group_size, const void* x_staged, const float* x_row_scale, int64_t rows_cap,
                      int dim, const int32_t* offsets, int n_experts, const void* w1, const void* w3, int inter,
                      int act, float limit, int round_gu, void* h_staged, float h_scale, int64_t n_rows,
                      void* stream);
int expert_tm_down(int wfmt, int group_size, const void* h_staged, float h_scale, int64_t rows_cap, int inter,
                   const int32_t* offsets, int n_experts, const void* w2, int dim, int round_o, float* o_rows,
                   int ldo, const int32_t* o_row_map, int64_t n_rows, void* stream,
                   const float* x_row_scale = nullptr);
// Dense (one-expert) down product split along K into k_splits fp32 partial slabs
// partials[s][n_rows][dim] (tm formats only; units of up to 128 rows); tm_down_splits picks
// the split count that fills the GPU without an empty split
int tm_down_splits(int inter, int dim, int64_t n_rows, int max_splits);
int expert_tm_down_split(int wfmt, int group_size, const void* h_staged, float h_scale, int64_t rows_cap,
                         int inter, const void* w2, int dim, int k_splits, float* partials, int64_t n_rows,
                         void* stream, const float* x_row_scale = nullptr);
// The streaming kernel's single-matrix product (f16, fp8) with K split into ranges, each
// writing an fp32 partial slab parts[split][n_rows][out_dim] in staged-row order: for a product
// whose row tiles alone would leave SMs idle or re-read each tile once per 8-64-row chunk.
// *splits_used = the ranges launched; 1: nothing was launched (another kernel fits better, or
// one range fills the GPU) and the caller runs the unsplit product.
int expert_stream_split(int wfmt, int group_size, const void* x_staged, const float* x_row_scale, int64_t rows_cap,
                        int k_dim, const int32_t* offsets, int n_groups, const void* w_packed, int out_dim,
                        int64_t n_rows, int max_splits, float* parts, void* stream, int* splits_used);
// h staging scale of the SwiGLU output: 1 when the clamp bounds |h| by limit^2, else 2^-8
float h_scale_for(int act, float limit);
// 0 = choose by rows per expert, 1 = always the decode kernel, 2 = tcgen05 where supported
int expert_regime();
// attention kernels: 0 = tensor-core kernels where they apply, 1 = CUDA-core kernels
int attn_kernel();

// Stage two row sets of the same x in one launch: rows of x in perm order (job a) and, when
// n_rows_b > 0, the first n_rows_b tokens in order (job b). Arguments as dsm_stage_rows.
int stage_rows_pair(const void* x, int x_dtype, int64_t n_tokens, int dim, const int32_t* perm, int64_t n_rows,
                    int topk, void* staged, int64_t rows_cap, float* row_scale, int64_t n_rows_b, void* staged_b,
                    int64_t rows_cap_b, float* row_scale_b, void* stream, const int32_t* n_valid = nullptr);

// Stage fp32 rows as two f16 rows each: row r the row itself (as dsm_stage_rows does), row
// n_rows + r the residual x - hi, with its own power-of-two scale, so that a product over both
// rows adds up to the fp32 row's product within ~2^-22. rows_cap >= dsm_stage_rows_cap(2 n_rows).
int stage_rows_hilo(const float* x, int64_t n_rows, int dim, void* staged, int64_t rows_cap, float* row_scale,
                    void* stream);

// ------------------------------------------------------------------------------------------
// geometry shared by staging, packing and the expert kernels
// ------------------------------------------------------------------------------------------
constexpr int kTileRows = 128;   // weight rows (output features) per work unit
constexpr int kChunkK = 128;     // K elements per pipeline stage / staging chunk
constexpr int kStagePitch = DSM_STAGE_PITCH;  // halves per staged row (128 + 32 pad)
constexpr int kPackHeader = 256; // bytes before the tiles in a packed weight buffer (>= 4*E)

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// bytes of one packed 128x128 tile (codes + per-tile metadata) per format
__host__ __device__ constexpr int tile_code_bytes(int wfmt) {
  return wfmt == DSM_WFMT_F16 ? 32768
         : (wfmt == DSM_WFMT_FP8_B128 || wfmt == DSM_WFMT_AFFINE8) ? 16384
                                                                     : 8192;
}
__host__ __device__ constexpr int tile_meta_bytes(int wfmt, int group_size) {
  return wfmt == DSM_WFMT_FP8_B128   ? 16
         : wfmt == DSM_WFMT_FP4_G32  ? 512
         : (wfmt == DSM_WFMT_AFFINE8 || wfmt == DSM_WFMT_AFFINE4)
             ? kTileRows * (kChunkK / (group_size > 0 ? group_size : 64)) * 4
             : 0;
}
__host__ __device__ constexpr int tile_bytes(int wfmt, int group_size) {
  return tile_code_bytes(wfmt) + tile_meta_bytes(wfmt, group_size);
}
inline int64_t packed_header_bytes(int n_experts) {
  return ceil_div(int64_t(n_experts) * 4, kPackHeader) * kPackHeader;
}

// ------------------------------------------------------------------------------------------
// device error word
// ------------------------------------------------------------------------------------------
extern __device__ int g_device_error;
__device__ __forceinline__ void raise_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

// ------------------------------------------------------------------------------------------
// PTX helpers: shared-memory addresses, mbarriers, bulk async copies, cache policies
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Wait for the phase with the given parity to complete, for at most ~2 s of wall time.
// Returns false (and records DSM_DEV_ERR_PIPELINE_TIMEOUT) if the budget ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > 2000000000ull) {
      raise_device_error(DSM_DEV_ERR_PIPELINE_TIMEOUT);
      return false;
    }
  }
}

// mbar_wait for a waiter that is off the critical path while it waits (epilogue warps that
// wait out a whole unit's main loop): between tries it sleeps ns, so its warps leave the issue
// slots to the converters and the MMA issuers. Same ~2 s bound.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, unsigned ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    __nanosleep(ns);
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > 2000000000ull) {
      raise_device_error(DSM_DEV_ERR_PIPELINE_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 1-D bulk copy global -> shared, completing `bytes` transaction bytes on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// ------------------------------------------------------------------------------------------
// code conversions (hardware cvt on sm_100a: exact for e4m3 / e2m1 into f16)
// ------------------------------------------------------------------------------------------
// 4 e4m3 bytes -> two f16x2: lo = (byte0, byte1), hi = (byte2, byte3) (low byte -> low half)
__device__ __forceinline__ void e4m3x4_to_f16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n .reg .b16 a, b;\n mov.b32 {a, b}, %2;\n cvt.rn.f16x2.e4m3x2 %0, a;\n cvt.rn.f16x2.e4m3x2 %1, b;\n}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}
// 8 e2m1 nibbles -> four f16x2: o[j] = (low nibble of byte j, high nibble of byte j)
__device__ __forceinline__ void e2m1x8_to_f16(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n .reg .b8 a, b, c, d;\n mov.b32 {a, b, c, d}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, a;\n cvt.rn.f16x2.e2m1x2 %1, b;\n"
      " cvt.rn.f16x2.e2m1x2 %2, c;\n cvt.rn.f16x2.e2m1x2 %3, d;\n}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}
// one e4m3 byte -> f16 (bits in the low half)
__device__ __forceinline__ uint32_t e4m3_to_f16_bits(uint32_t byte) {
  uint32_t lo, hi;
  e4m3x4_to_f16(byte & 0xFFu, lo, hi);
  return lo & 0xFFFFu;
}
// bytes 0,1 (resp. 2,3) of w placed as f16 (1024 + byte): magic-number conversion of uint8
__device__ __forceinline__ void u8x4_to_f16_plus1024(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = __byte_perm(w, 0x64646464u, 0x4140);
  hi = __byte_perm(w, 0x64646464u, 0x4342);
}
// nibbles (j, j+4) of w as f16 (1024 + nibble), j = 0..3
__device__ __forceinline__ void u4x8_to_f16_plus1024(uint32_t w, uint32_t (&o)[4]) {
  o[0] = (w & 0x000F000Fu) | 0x64006400u;
  o[1] = ((w >> 4) & 0x000F000Fu) | 0x64006400u;
  o[2] = ((w >> 8) & 0x000F000Fu) | 0x64006400u;
  o[3] = ((w >> 12) & 0x000F000Fu) | 0x64006400u;
}
__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Sigmoid of the expert activations: the hardware exp2 and reciprocal approximations (a few
// fp32 ulps, far below the bf16 rounding that follows in most paths). The correctly rounded
// reciprocal (or an IEEE 1/x) is a long instruction sequence and made the SwiGLU epilogues
// latency-bound. Routing scores and the hyper-connection mixes keep expf and IEEE division.
__device__ __forceinline__ float act_sigmoid(float v) { return __fdividef(1.f, 1.f + __expf(-v)); }

// SwiGLU of the expert products (dspark_mlx/model/moe.py:37-44): silu(g) * u, with g clamped
// above and u on both sides at `limit` when limit > 0. DSM_ACT_SILU_MUL_BF16 is nn.silu(g) * u
// on bf16 arrays, where every elementwise op rounds to bf16. The kind is a compile-time
// parameter and the clamp a select, so a loop over columns has no branch.
template <bool kSiluBf16>
__device__ __forceinline__ float swiglu(float g, float u, float limit) {
  if constexpr (kSiluBf16) {
    const float sig = bf16_round(act_sigmoid(g));
    return bf16_round(g * sig) * u;
  } else {
    const bool clamp = limit > 0.f;
    u = clamp ? fminf(fmaxf(u, -limit), limit) : u;
    g = clamp ? fminf(g, limit) : g;
    return g * act_sigmoid(g) * u;
  }
}
__device__ __forceinline__ float swiglu(float g, float u, int act, float limit) {
  return act == DSM_ACT_SILU_MUL_BF16 ? swiglu<true>(g, u, limit) : swiglu<false>(g, u, limit);
}

template <typename T>
__device__ __forceinline__ float load_as_float(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_as_float<float>(const float* p, int64_t i) {
  return p[i];
}
template <>
__device__ __forceinline__ float load_as_float<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

// Activations of the attention paths are fp32 or bf16 (T): loads to fp32, stores from fp32,
// and an fp32 value rounded to T as the reference's arrays of dtype T hold it.
template <typename T>
__device__ __forceinline__ float ld_f(const T* p, int64_t i) {
  if constexpr (std::is_same<T, float>::value)
    return p[i];
  else
    return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ T st_f(float v) {
  if constexpr (std::is_same<T, float>::value)
    return v;
  else
    return __float2bfloat16_rn(v);
}
template <typename T>
__device__ __forceinline__ float rnd(float v) {
  if constexpr (std::is_same<T, float>::value)
    return v;
  else
    return __bfloat162float(__float2bfloat16_rn(v));
}

}  // namespace dsm
