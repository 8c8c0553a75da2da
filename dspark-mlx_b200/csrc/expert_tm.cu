// Grouped expert products for fp4 experts (e2m1 codes, e4m3 scale per 32 K, fp32 per-expert
// tensor scale; dspark_mlx/loading.py:110-114 dequantisation) and MLX affine 8/4-bit experts
// (MoE.quantize, dspark_mlx/model/moe.py:124-130, and the Qwen3 MLP's QuantizedLinears),
// applied inside the products of dspark_mlx/model/moe.py:132-149, at every token count: the
// weights are dequantised in registers straight into tensor memory and multiplied there by
// tcgen05.
//
// Work unit = (expert e, 128 weight rows, up to BN of the expert's staged rows). Persistent
// CTAs (one per SM), warp-specialised:
//   warps 0-3   epilogue: tcgen05.ld of the accumulators (warp w reads TMEM lanes 32w..),
//               per-expert tensor scale and activation row scale, SwiGLU (gate/up) or
//               output rows (down);
//   warp 4      producer: per 128-K stage, one bulk copy of each packed 8.5 KB weight tile
//               (codes + group scales) and TMA loads of the unit's activation rows (16-row
//               boxes of 64 f16, 128-byte swizzle) into a ring of shared-memory stages;
//   warps 8-15  converters: each thread owns one weight row (its TMEM lane) and a K range of
//               the stage, read with ld.shared.v4 (16 bytes per chunk), converted and
//               written into the A buffer with tcgen05.st:
//                 fp4    hardware e2m1 -> f16 conversion, one f16 multiply by the group
//                        scale (exact: at most 6 significant bits);
//                 affine magic-number uint8 / uint4 -> f16, then one f16 fma with the
//                        group's scale and bias, both pre-multiplied at pack time by the
//                        expert's power-of-two prescale (max |w| -> [2^14, 2^15)); the
//                        epilogue undoes the prescale. One f16 rounding of each weight,
//                        2^-11 relative, where MLX dequantises in fp32;
//   warps 16..  P MMA issuers (one thread each): tcgen05.mma kind::f16, M = 128, N = the
//               unit's rows rounded up to 16, A read from TMEM, B (activations) from shared
//               memory. One thread issues at most one such MMA every ~46 cycles whatever N
//               is, so the 8 x (gate, up) MMAs of a stage are split over P threads, each
//               accumulating its share of the k16 steps of one matrix into its own partial
//               D in TMEM (two buffers where TMEM allows, so an epilogue overlaps the next
//               unit); the epilogue adds the partials.
// The activations are read by the tensor core from shared memory, so no register traffic or
// legacy MMA pipe is spent on them; the ALU work per weight byte is the conversion alone.
//
// Packed tiles (128 rows x 128 K, written by dsm_pack_weights): codes [16-byte chunk][row]
// [16 bytes] (fp4 and 4-bit affine: 32 K per chunk; 8-bit affine: 16 K), then the scales:
// fp4 e4m3 [row][32-K group]; affine f16 (scale, bias) pairs [row][group]. A warp's
// ld.shared.v4 of one chunk covers 32 consecutive rows: 512 contiguous bytes, no bank
// conflicts.
#include <algorithm>
#include <type_traits>

#include "tcgen05.cuh"

namespace dsm {
namespace {

using namespace tc;

constexpr int kTmM = 128;
constexpr int kTmEpiWarps = 4;    // warps 0-3
constexpr int kTmProducer = 4;
constexpr int kTmConv0 = 8;       // first converter warp (a multiple of 4: warp % 4 = TMEM sub-partition)
constexpr int kTmBoxRows = 16;

// PAIR: the single-matrix (down) product over two adjacent row tiles per unit, built like the
// gate/up pair (two A matrices, one activation tile per stage feeding both), so each staged
// activation tile serves 256 weight rows instead of 128.
template <int FMT, bool DUAL, int BN, int CW, int P, bool PAIR = false>
struct TmCfg {
  static_assert(!(DUAL && PAIR), "PAIR is the single-matrix product");
  static constexpr bool kAffine = FMT != DSM_WFMT_FP4_G32;
  static constexpr bool kB8 = FMT == DSM_WFMT_AFFINE8;
  static constexpr int kCodeBytes = kB8 ? 16384 : 8192;
  static constexpr int kChunkK = kB8 ? 16 : 32;         // K per 16-byte chunk
  static constexpr int kRowChunks = 128 / kChunkK;      // chunks per row of a tile
  static constexpr int NM = (DUAL || PAIR) ? 2 : 1;
  // 128-K chunks per stage: two for the single-matrix (down) product, whose tiles carry half
  // the bytes of a gate/up pair, so the per-stage barrier, copy and commit costs are spread
  // over the same bytes; the gate/up pair keeps one (its A buffer is already 128 columns),
  // and so do 128-row units, whose activation rows alone fill 32 KB per chunk
  static constexpr int KS = (DUAL || PAIR || BN >= 128) ? 1 : 2;
  static constexpr int kMma0 = kTmConv0 + CW;  // first MMA issuer warp
  static constexpr int kThreads = 32 * (kMma0 + P);
  static constexpr int kKkStride = P / NM;     // issuer p: matrix p % NM, k16 steps p / NM + j * kKkStride
  static constexpr int kBHalf = BN * 128;    // one 64-K half of the activation rows
  static constexpr int kOffRaw = 2 * KS * kBHalf;
  static constexpr int kACols = NM * KS * 64;  // one A buffer: KS x 128 K of f16 per matrix
  // accumulator buffers of P partials each: two (an epilogue overlaps the next unit's MMAs)
  // when they fit beside two A buffers in the 512 TMEM columns, else one
  static constexpr int DB = (2 * P * BN + 2 * kACols <= 512) ? 2 : 1;
  static constexpr int kDCols = DB * P * BN;
  static constexpr int kSteps = 8 * KS / kKkStride;  // k16 steps of one issuer per full stage
  static constexpr int kABufs = std::min(4, (512 - kDCols) / kACols);
  static constexpr int kParts = CW / 4;            // converter warps per TMEM sub-partition
  static constexpr int kChunks = kRowChunks / kParts;  // chunks per converter thread per matrix
  static constexpr int kCols = kChunks * kChunkK / 2;  // TMEM columns per converter thread per matrix
  static_assert(CW == 8 || CW == 16, "converter warps");
  static_assert(P % NM == 0 && 8 % (P / NM) == 0, "issuers split the k16 steps evenly");
  static_assert(kABufs >= 2, "TMEM budget");
  static_assert(kCols == 16 || kCols == 32, "converter store width");
};

// shared-memory stage: [activation rows: KS chunks x 2 x 64-K halves][packed tile x KS x NM],
// 1024-aligned
inline int tm_stage_bytes(int off_raw, int tiles, int tile_b) { return (off_raw + tiles * tile_b + 1023) / 1024 * 1024; }

struct TmArgs {
  const uint8_t* wa;
  const uint8_t* wb;
  const float* act_scale;
  float act_scale_const;
  const int32_t* offsets;
  int64_t n_rows;
  int n_experts;
  int out_rows;
  int rt_count;
  int kc_count;
  int group_size;  // affine
  int tile_b;      // packed tile bytes
  int stage_b;     // shared-memory stage bytes
  int k_splits;    // single-matrix product only: K ranges per row tile, each writing its own
                   // fp32 partial slab (o_out + split * o_split_stride); 1 = no split
  int k_per;       // 128-K chunks per split, a multiple of KS
  int64_t o_split_stride;
  int act;
  float limit;
  int round_gu;
  float h_scale;
  __half* h_out;
  int64_t h_rows_cap;
  float* o_out;
  const int32_t* o_row_map;
  int ldo;
  int round_o;
};

__device__ __forceinline__ int tm_first(const TmArgs& a, int e) { return a.offsets ? a.offsets[e] : 0; }
__device__ __forceinline__ int tm_count(const TmArgs& a, int e) {
  return a.offsets ? a.offsets[e + 1] - a.offsets[e] : int(a.n_rows);
}
__device__ __forceinline__ int tm_find(const int* pre, int n, int u);

// Work unit u: expert e, weight row tile rt, block `chunk` of the expert's rows, K split ks
// covering 128-K chunks [kc0, kc1). Units of one row tile are adjacent, token blocks
// innermost, so the CTAs re-reading a weight tile for other token blocks run together.
struct TmUnit {
  int e, rt, chunk, ks, kc0, kc1, cnt;
};
template <int BN>
__device__ __forceinline__ TmUnit tm_unit(const TmArgs& a, const int* pre, int E, int u, int kcs) {
  TmUnit w;
  w.e = tm_find(pre, E, u);
  w.cnt = tm_count(a, w.e);
  const int nch = (w.cnt + BN - 1) / BN;
  const int per_rt = nch * a.k_splits;
  const int local = u - pre[w.e];
  w.rt = local / per_rt;
  const int r2 = local % per_rt;
  w.ks = r2 / nch;
  w.chunk = r2 % nch;
  w.kc0 = w.ks * a.k_per;
  w.kc1 = min(kcs, w.kc0 + a.k_per);
  return w;
}

__device__ __forceinline__ int tm_find(const int* pre, int n, int u) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (pre[mid] <= u)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

template <int FMT, bool DUAL, int BN, int CW, int P, bool PAIR = false>
__global__ void __launch_bounds__(TmCfg<FMT, DUAL, BN, CW, P, PAIR>::kThreads, 1)
    expert_tm_kernel(const TmArgs a, const __grid_constant__ CUtensorMap xmap, int n_stages) {
  using C = TmCfg<FMT, DUAL, BN, CW, P, PAIR>;
  constexpr int NM = C::NM, NA = C::kABufs;
  const int S = n_stages;
  const int stage_b = a.stage_b, tile_b = a.tile_b;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base - raw0);
  uint64_t* full = reinterpret_cast<uint64_t*>(sbase + S * stage_b);
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;
  uint64_t* tfull = afull + NA;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* pre = const_cast<int*>(reinterpret_cast<volatile int*>(tmem_slot + 2));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.n_experts;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      // converters done reading the codes + MMAs done reading B and the stage's A buffer
      mbar_init(&empty[s], CW + P);
    }
    for (int b = 0; b < NA; ++b) mbar_init(&afull[b], CW);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], P);
      mbar_init(&tempty[b], kTmEpiWarps);
    }
    mbar_init(drain, P);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == C::kMma0) tmem_alloc(tmem_slot, 512);
  if (warp == kTmProducer) {  // units per expert: rt_count x ceil(count / BN), scanned into pre[1..E]
    int carry = 0;
    if (lane == 0) pre[0] = 0;
    for (int b0 = 0; b0 < E; b0 += 32) {
      const int e = b0 + lane;
      int v = 0;
      if (e < E) {
        const int cnt = tm_count(a, e);
        v = cnt > 0 ? (PAIR ? a.rt_count / 2 : a.rt_count) * ((cnt + BN - 1) / BN) * a.k_splits : 0;
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = pre[E];
  const int64_t hdr_bytes = ceil_div(int64_t(E) * 4, kPackHeader) * kPackHeader;
  const uint8_t* tiles_a = a.wa + hdr_bytes;
  const uint8_t* tiles_b = DUAL ? a.wb + hdr_bytes : nullptr;
  const int kcs = a.kc_count;

  // Epilogue of the CTA's j-th unit u for TMEM sub-partition sp: its 16-column blocks part,
  // part + nparts, ... . The epilogue warps take every unit; the converter warps, idle once
  // their last stage is written, take a share of the CTA's last unit (the whole epilogue when
  // a CTA has one unit, as the dense layers' wide units do). False on abort.
  auto epilogue_unit = [&](int j, int u, int sp, int part, int nparts) -> bool {
    const int rloc = 32 * sp + lane;
    const uint32_t lane_base = tmem + (uint32_t(32 * sp) << 16);
    const TmUnit w = tm_unit<BN>(a, pre, E, u, kcs);
    const int e = w.e, rt = w.rt, chunk = w.chunk;
    const int off = tm_first(a, e);
    const int rows = min(BN, w.cnt - chunk * BN);
    float* const o_out = a.o_out + w.ks * a.o_split_stride;
    const int buf = j % C::DB;
    if (*abort_flag || !mbar_wait_backoff(&tfull[buf], (j / C::DB) & 1, 200)) {
      *abort_flag = 1;
      return false;
    }
    tc_fence_after();
    const float wmul_a = reinterpret_cast<const float*>(a.wa)[e];
    const float wmul_b = DUAL ? reinterpret_cast<const float*>(a.wb)[e] : 1.f;
    for (int cb = 16 * part; cb < rows; cb += 16 * nparts) {
      // partial accumulators, added in issuer order: issuer q holds matrix q % NM
      float gsum[16], usum[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) gsum[i] = usum[i] = 0.f;
#pragma unroll
      for (int q = 0; q < P; ++q) {
        uint32_t pv[16];
        tmem_ld16(lane_base + uint32_t((buf * P + q) * BN + cb), pv);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (q % NM == 0)
            gsum[i] += __uint_as_float(pv[i]);
          else
            usum[i] += __uint_as_float(pv[i]);
        }
      }
      if constexpr (DUAL && P >= 4) {
        // decode widths: the epilogue overlaps the next unit's main loop (two accumulator
        // buffers), and the branch-free form below would not fit the register budget of
        // this thread count
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int col = cb + i;
          if (col >= rows) break;
          const int64_t r = int64_t(off) + chunk * BN + col;
          const float xs = a.act_scale ? a.act_scale[r] : a.act_scale_const;
          float gg = gsum[i] * xs * wmul_a;
          float uu = usum[i] * xs * wmul_b;
          if (a.round_gu & 1) {
            gg = bf16_round(gg);
            uu = bf16_round(uu);
          }
          float h = swiglu(gg, uu, a.act, a.limit);
          if (a.round_gu & 2) h = bf16_round(h);
          a.h_out[(int64_t(rt) * a.h_rows_cap + r) * kStagePitch + rloc] = __float2half_rn(h * a.h_scale);
        }
        continue;
      }
      if constexpr (PAIR) {
        // the pair's two row tiles, 2 rt and 2 rt + 1: the partials of matrix m are row tile
        // 2 rt + m's outputs
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int col = cb + i;
          if (col >= rows) break;
          const int64_t r = int64_t(off) + chunk * BN + col;
          const float xs = a.act_scale ? a.act_scale[r] : a.act_scale_const;
          const int64_t orow = a.o_row_map ? int64_t(a.o_row_map[r]) : r;
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const int d = (2 * rt + m) * kTmM + rloc;
            float v = (m ? usum[i] : gsum[i]) * xs * wmul_a;
            v = a.round_o ? bf16_round(v) : v;
            if (d < a.out_rows) o_out[orow * a.ldo + d] = v;
          }
        }
        continue;
      }
      // the block's 16 row scales (and output rows): one guarded load per lane, broadcast
      // with a constant source lane per column
      const int cl = cb + (lane & 15);
      const int rl = off + chunk * BN + cl;
      const float xs_b = (cl < rows && a.act_scale) ? a.act_scale[rl] : a.act_scale_const;
      if constexpr (DUAL) {
        // all 16 columns are computed without a branch (columns past `rows` hold unused
        // accumulators), so their activation chains interleave; only the stores are guarded
        const bool rg = a.round_gu & 1, rh = a.round_gu & 2;
        __half* hp = a.h_out + (int64_t(rt) * a.h_rows_cap + off + chunk * BN + cb) * kStagePitch + rloc;
        auto block = [&](auto silu_tag) {
#pragma unroll
          for (int i0 = 0; i0 < 16; i0 += 8) {  // 8 chains at a time: ILP within the register budget
            float hv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float xs = __shfl_sync(0xffffffffu, xs_b, i0 + i);
              float gg = gsum[i0 + i] * xs * wmul_a;
              float uu = usum[i0 + i] * xs * wmul_b;
              gg = rg ? bf16_round(gg) : gg;
              uu = rg ? bf16_round(uu) : uu;
              const float h = swiglu<decltype(silu_tag)::value>(gg, uu, a.limit);
              hv[i] = (rh ? bf16_round(h) : h) * a.h_scale;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (cb + i0 + i < rows) hp[int64_t(i0 + i) * kStagePitch] = __float2half_rn(hv[i]);
          }
        };
        if (a.act == DSM_ACT_SILU_MUL_BF16)
          block(std::true_type{});
        else
          block(std::false_type{});
      } else {
        const int or_b = (cl < rows && a.o_row_map) ? a.o_row_map[rl] : rl;
        const int d = rt * kTmM + rloc;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float xs = __shfl_sync(0xffffffffu, xs_b, i);
          const int orow = __shfl_sync(0xffffffffu, or_b, i);
          float v = gsum[i] * xs * wmul_a;
          v = a.round_o ? bf16_round(v) : v;
          if (cb + i < rows && d < a.out_rows) o_out[int64_t(orow) * a.ldo + d] = v;
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    return true;
  };

  if (warp == kTmProducer) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const TmUnit w = tm_unit<BN>(a, pre, E, u, kcs);
        const int row0 = tm_first(a, w.e) + w.chunk * BN;
        const int nbox = (min(BN, w.cnt - w.chunk * BN) + kTmBoxRows - 1) / kTmBoxRows;
        // first row tile: the unit's (gate/up: both matrices'), or the pair's first (PAIR)
        const int64_t tile0 = (int64_t(w.e) * a.rt_count + (PAIR ? 2 * w.rt : w.rt)) * kcs;
        const uint32_t tx1 = uint32_t(NM * tile_b + 2 * nbox * kTmBoxRows * 128);  // per chunk
        for (int kc = w.kc0; kc < w.kc1; kc += C::KS) {
          const int nk = min(C::KS, w.kc1 - kc);
          if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* st = sbase + s * stage_b;
          mbar_arrive_expect_tx(&full[s], uint32_t(nk) * tx1);
          for (int j = 0; j < nk; ++j) {
            uint8_t* raw = st + C::kOffRaw + j * NM * tile_b;
            bulk_g2s(raw, tiles_a + (tile0 + kc + j) * tile_b, uint32_t(tile_b), &full[s], pol_w);
            if (DUAL) bulk_g2s(raw + tile_b, tiles_b + (tile0 + kc + j) * tile_b, uint32_t(tile_b), &full[s], pol_w);
            if (PAIR)
              bulk_g2s(raw + tile_b, tiles_a + (tile0 + kcs + kc + j) * tile_b, uint32_t(tile_b), &full[s], pol_w);
            for (int h = 0; h < 2; ++h)
              for (int b = 0; b < nbox; ++b)
                tma_load_3d(smem_u32(st + (2 * j + h) * C::kBHalf + b * kTmBoxRows * 128), &xmap, h * 64,
                            row0 + b * kTmBoxRows, kc + j, &full[s]);
          }
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok)
        for (int i = 0; i < 100; ++i) __nanosleep(1000);
    }
  } else if (warp >= C::kMma0) {
    // ------------------------------------------------------------------ MMA issuers
    const int p = warp - C::kMma0;
    const int m = p % NM, kk0 = p / NM;
    if (lane == 0) {
      int s = 0, ab = 0;
      uint32_t aph = 0;
      bool ok = true;
      int j = 0;
      // descriptors and TMEM addresses, precomputed: one add per MMA in the loop
      const uint64_t bdesc0 = umma_desc_sw128(smem_u32(sbase));
      constexpr int kSteps = C::kSteps;
      uint64_t boff[kSteps];
      uint32_t aoff[kSteps];
#pragma unroll
      for (int i = 0; i < kSteps; ++i) {
        const int kk = kk0 + i * C::kKkStride;  // k16 step of the stage: chunk kk / 8, half (kk % 8) / 4
        boff[i] = uint64_t(((kk >> 2) * C::kBHalf + (kk & 3) * 32) >> 4);
        aoff[i] = uint32_t(C::kDCols + m * 64 * C::KS + kk * 8);
      }
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++j) {
        const TmUnit w = tm_unit<BN>(a, pre, E, u, kcs);
        const int n_mma = (min(BN, w.cnt - w.chunk * BN) + 15) / 16 * 16;
        const uint32_t idesc = umma_idesc_f16(kTmM, n_mma);
        const int buf = j % C::DB;
        if (*abort_flag || !mbar_wait(&tempty[buf], ((j / C::DB) & 1) ^ 1u)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t((buf * P + p) * BN);
        for (int kc = w.kc0; kc < w.kc1; kc += C::KS) {
          const int nkk = 8 * min(C::KS, w.kc1 - kc);  // k16 steps in this stage
          // the converters arrive on afull only after they saw the stage's copies land
          // (full[s]), so acquiring afull also orders the activation rows read below
          if (*abort_flag || !mbar_wait(&afull[ab], aph)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bst = bdesc0 + uint64_t((s * stage_b) >> 4);
          const uint32_t ast = tmem + uint32_t(ab * C::kACols);
#pragma unroll
          for (int i = 0; i < kSteps; ++i) {
            if (kk0 + i * C::kKkStride >= nkk) break;
            umma_f16_tmem_a(d, ast + aoff[i], bst + boff[i], idesc, (kc > w.kc0 || i > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);  // activation rows and the A buffer read
          if (++s == S) s = 0;
          if (++ab == NA) {
            ab = 0;
            aph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
      umma_commit(drain);  // every MMA of this thread completes before TMEM is released
      mbar_wait(drain, 0);
    }
  } else if (warp >= kTmConv0) {
    // ------------------------------------------------------------------ converters
    const int sp = warp & 3;                     // TMEM sub-partition: lanes 32*sp ..
    const int part = (warp - kTmConv0) >> 2;     // K range of the stage: chunks part*kChunks ..
    const int row = 32 * sp + lane;              // weight row = TMEM lane
    const uint32_t lane_base = tmem + (uint32_t(32 * sp) << 16);
    // A buffer ab of stage g is free once the MMAs of stage g - NA completed: the empty
    // barrier of that stage's slot (ws) in the phase of its lap (wph). That barrier cannot
    // run a phase ahead: its next phase needs these converters' arrivals for a later stage.
    int s = 0, ab = 0, g = 0, ws = 0;
    uint32_t ph = 0, wph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
      const TmUnit w = tm_unit<BN>(a, pre, E, u, kcs);
      for (int kc = w.kc0; kc < w.kc1; kc += C::KS, ++g) {
        const int nk = min(C::KS, w.kc1 - kc);
        if (*abort_flag || !mbar_wait(&full[s], ph)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        if (g >= NA) {
          if (*abort_flag || !mbar_wait(&empty[ws], wph)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          if (++ws == S) {
            ws = 0;
            wph ^= 1u;
          }
        }
        tc_fence_after();
        const uint32_t st = smem_u32(sbase + s * stage_b) + C::kOffRaw;
#pragma unroll
        for (int jm = 0; jm < C::KS * NM; ++jm) {
          const int j = jm / NM, m = jm % NM;  // chunk of the stage, matrix
          if (j >= nk) break;
          const uint32_t raw = st + jm * tile_b;
          const uint32_t meta = raw + C::kCodeBytes;
          uint32_t out[C::kCols];
          if constexpr (!C::kAffine) {
            const uint32_t sw = lds32(meta + row * 4);  // e4m3 scales of the row's 4 groups
            uint32_t sp_lo, sp_hi;  // the 4 scales as f16 pairs: two conversions per row and stage
            e4m3x4_to_f16(sw, sp_lo, sp_hi);
#pragma unroll
            for (int c = 0; c < C::kChunks; ++c) {
              const int cc = part * C::kChunks + c;
              const uint4 v = lds128(raw + (cc * kTmM + row) * 16);
              const uint32_t sp = (cc >> 1) ? sp_hi : sp_lo;
              const uint32_t s2 = __byte_perm(sp, 0, (cc & 1) ? 0x3232 : 0x1010);
              const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int wi = 0; wi < 4; ++wi) {
                uint32_t o[4];
                e2m1x8_to_f16(w4[wi], o);
#pragma unroll
                for (int t = 0; t < 4; ++t) out[16 * c + 4 * wi + t] = hmul2_bits(o[t], s2);
              }
            }
          } else {
            const uint32_t magic = 0x64006400u;  // f16x2 (1024, 1024)
            const int gpt = kChunkK / a.group_size;  // groups per tile row
#pragma unroll
            for (int c = 0; c < C::kChunks; ++c) {
              const int cc = part * C::kChunks + c;
              const uint32_t sb = lds32(meta + (row * gpt + (cc * C::kChunkK) / a.group_size) * 4);
              const uint32_t s2 = __byte_perm(sb, 0, 0x1010), b2 = __byte_perm(sb, 0, 0x3232);
              const uint4 v = lds128(raw + (cc * kTmM + row) * 16);
              const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int wi = 0; wi < 4; ++wi) {
                if constexpr (C::kB8) {  // bytes j, j+1 are one K pair
                  uint32_t lo, hi;
                  u8x4_to_f16_plus1024(w4[wi], lo, hi);
                  out[8 * c + 2 * wi] = hfma2_bits(hsub2_bits(lo, magic), s2, b2);
                  out[8 * c + 2 * wi + 1] = hfma2_bits(hsub2_bits(hi, magic), s2, b2);
                } else {  // nibbles i, i+4 are one K pair
                  uint32_t o[4];
                  u4x8_to_f16_plus1024(w4[wi], o);
#pragma unroll
                  for (int t = 0; t < 4; ++t) out[16 * c + 4 * wi + t] = hfma2_bits(hsub2_bits(o[t], magic), s2, b2);
                }
              }
            }
          }
          const uint32_t col = uint32_t(C::kDCols + ab * C::kACols + (m * C::KS + j) * 64 + part * C::kCols);
          if constexpr (C::kCols == 32)
            tmem_st32(lane_base + col, out);
          else
            tmem_st16(lane_base + col, out);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&afull[ab]);
          mbar_arrive(&empty[s]);
        }
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
        if (++ab == NA) ab = 0;
      }
    }
    // this warp's share of the CTA's last unit's epilogue
    if (ok && int(blockIdx.x) < total) {
      const int j = (total - 1 - int(blockIdx.x)) / int(gridDim.x);
      epilogue_unit(j, int(blockIdx.x) + j * int(gridDim.x), warp & 3, 1 + part, 1 + CW / 4);
    }
  } else if (warp < kTmEpiWarps) {
    // ------------------------------------------------------------------ epilogue
    int j = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++j) {
      const bool last = u + int(gridDim.x) >= total;
      if (!epilogue_unit(j, u, warp, 0, last ? 1 + CW / 4 : 1)) break;
      if (lane == 0) mbar_arrive(&tempty[j % C::DB]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == C::kMma0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int FMT, bool DUAL, int BN, int CW, int P, bool PAIR = false>
int launch_tm(TmArgs a, const void* staged, int64_t rows_cap, cudaStream_t stream) {
  using C = TmCfg<FMT, DUAL, BN, CW, P, PAIR>;
  CUtensorMap map;
  if (int rc = make_stage_map(&map, staged, rows_cap, a.kc_count, kTmBoxRows)) return rc;
  a.tile_b = tile_bytes(FMT, a.group_size);
  a.stage_b = tm_stage_bytes(C::kOffRaw, C::NM * C::KS, a.tile_b);
  const int n_stages = std::min(8, (200 * 1024) / a.stage_b);
  if (n_stages < 2) return fail(DSM_ERR_UNSUPPORTED, "expert_tm: tile too large for the shared-memory ring");
  const size_t smem = 1024 + size_t(n_stages) * a.stage_b + 8 * (2 * n_stages + C::kABufs + 5) + 16 +
                      size_t(a.n_experts + 1) * 4;
  auto kern = expert_tm_kernel<FMT, DUAL, BN, CW, P, PAIR>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return check_launch("expert_tm smem attribute");
  kern<<<persistent_ctas(), C::kThreads, smem, stream>>>(a, map, n_stages);
  return check_launch("expert_tm");
}

constexpr int kTmCW = 8;

// Unit width: decode draft blocks put a few rows on each expert (units of up to 32 rows,
// four MMA issuers splitting each stage's k16 steps); from an average of 32 rows per busy
// expert (a dense layer run as one expert, prefill) units of up to 64 rows with two
// issuers convert each weight tile half as often -- as long as they still give every SM a
// unit (a product with few row tiles keeps the narrower units). Both keep two accumulator
// buffers of P x BN = 128 TMEM columns.
// A dense layer's gate/up pair run as one expert (rows of 100+ tokens) takes units of up to
// 128 rows when they fit in one wave: each SM then converts its weight tiles once, and the
// single accumulator buffer this width leaves room for costs nothing with one unit per SM.
// (The down product keeps narrower units: its two-chunk stages of 128 rows would leave two
// stages in flight, and it has few row tiles to spread.)
template <int FMT, bool DUAL>
int launch_width(const TmArgs& a, const void* staged, int64_t rows_cap, cudaStream_t s) {
  if constexpr (!DUAL) {
    // K-split dense products: every weight tile converted once, for up to 128 rows at a time
    if (a.k_splits > 1) return launch_tm<FMT, DUAL, 128, kTmCW, 2>(a, staged, rows_cap, s);
  }
  const int64_t busy = std::max<int64_t>(1, std::min<int64_t>(a.n_rows, a.n_experts));
  const int64_t units64 = int64_t(a.rt_count) * (busy + a.n_rows / 64);  // estimates
  const int64_t units128 = int64_t(a.rt_count) * (busy + a.n_rows / 128);
  if constexpr (DUAL) {
    if (a.n_rows > 96 * busy && units128 <= persistent_ctas())
      return launch_tm<FMT, DUAL, 128, kTmCW, 2>(a, staged, rows_cap, s);
  }
  // the down product in row-tile pairs where the tiles pair up: each staged activation tile
  // then feeds 256 weight rows, as in the gate/up pair, instead of 128
  const bool pair = !DUAL && a.k_splits <= 1 && a.rt_count % 2 == 0;
  if (a.n_rows > 32 * busy && units64 >= persistent_ctas()) {
    if (pair) return launch_tm<FMT, DUAL, 64, kTmCW, 2, !DUAL>(a, staged, rows_cap, s);
    return launch_tm<FMT, DUAL, 64, kTmCW, 2>(a, staged, rows_cap, s);
  }
  if (pair) return launch_tm<FMT, DUAL, 32, kTmCW, 4, !DUAL>(a, staged, rows_cap, s);
  return launch_tm<FMT, DUAL, 32, kTmCW, 4>(a, staged, rows_cap, s);
}

template <bool DUAL>
int dispatch_tm(int wfmt, const TmArgs& a, const void* staged, int64_t rows_cap, cudaStream_t s) {
  switch (wfmt) {
    case DSM_WFMT_FP4_G32: return launch_width<DSM_WFMT_FP4_G32, DUAL>(a, staged, rows_cap, s);
    case DSM_WFMT_AFFINE8: return launch_width<DSM_WFMT_AFFINE8, DUAL>(a, staged, rows_cap, s);
    case DSM_WFMT_AFFINE4: return launch_width<DSM_WFMT_AFFINE4, DUAL>(a, staged, rows_cap, s);
    default: return fail(DSM_ERR_INVALID_ARGUMENT, "expert_tm: format not handled by the tensor-memory kernel");
  }
}

}  // namespace

bool tm_supports(int wfmt) {
  return wfmt == DSM_WFMT_FP4_G32 || wfmt == DSM_WFMT_AFFINE8 || wfmt == DSM_WFMT_AFFINE4;
}

int expert_tm_gate_up(int wfmt, int group_size, const void* x_staged, const float* x_row_scale, int64_t rows_cap,
                      int dim, const int32_t* offsets, int n_experts, const void* w1, const void* w3, int inter,
                      int act, float limit, int round_gu, void* h_staged, float h_scale, int64_t n_rows,
                      void* stream) {
  TmArgs a{};
  a.wa = static_cast<const uint8_t*>(w1);
  a.wb = static_cast<const uint8_t*>(w3);
  a.act_scale = x_row_scale;
  a.act_scale_const = 1.f;
  a.offsets = offsets;
  a.n_rows = n_rows;
  a.n_experts = n_experts;
  a.out_rows = inter;
  a.rt_count = int(ceil_div(inter, kTmM));
  a.kc_count = int(ceil_div(dim, kChunkK));
  a.act = act;
  a.limit = limit;
  a.round_gu = round_gu;
  a.h_scale = h_scale;
  a.h_out = static_cast<__half*>(h_staged);
  a.h_rows_cap = rows_cap;
  a.group_size = group_size > 0 ? group_size : 64;
  a.k_splits = 1;
  a.k_per = a.kc_count;
  return dispatch_tm<true>(wfmt, a, x_staged, rows_cap, as_stream(stream));
}

int expert_tm_down(int wfmt, int group_size, const void* h_staged, float h_scale, int64_t rows_cap, int inter,
                   const int32_t* offsets, int n_experts, const void* w2, int dim, int round_o, float* o_rows,
                   int ldo, const int32_t* o_row_map, int64_t n_rows, void* stream, const float* x_row_scale) {
  TmArgs a{};
  a.wa = static_cast<const uint8_t*>(w2);
  a.wb = nullptr;
  a.act_scale = x_row_scale;
  a.act_scale_const = x_row_scale ? 1.f : 1.f / h_scale;
  a.offsets = offsets;
  a.n_rows = n_rows;
  a.n_experts = n_experts;
  a.out_rows = dim;
  a.rt_count = int(ceil_div(dim, kTmM));
  a.kc_count = int(ceil_div(inter, kChunkK));
  a.o_out = o_rows;
  a.o_row_map = o_row_map;
  a.ldo = ldo;
  a.round_o = round_o;
  a.group_size = group_size > 0 ? group_size : 64;
  a.k_splits = 1;
  a.k_per = a.kc_count;
  return dispatch_tm<false>(wfmt, a, h_staged, rows_cap, as_stream(stream));
}

int tm_down_splits(int inter, int dim, int64_t n_rows, int max_splits) {
  const int kcs = int(ceil_div(inter, kChunkK));
  const int64_t units = ceil_div(dim, kTmM) * ceil_div(n_rows, 128);
  int sp = int(std::min<int64_t>(std::min(max_splits, kcs), std::max<int64_t>(1, persistent_ctas() / units)));
  if (sp <= 1) return 1;
  const int per = (kcs + sp - 1) / sp;
  return (kcs + per - 1) / per;  // no empty split
}

int expert_tm_down_split(int wfmt, int group_size, const void* h_staged, float h_scale, int64_t rows_cap,
                         int inter, const void* w2, int dim, int k_splits, float* partials, int64_t n_rows,
                         void* stream, const float* x_row_scale) {
  TmArgs a{};
  a.wa = static_cast<const uint8_t*>(w2);
  a.wb = nullptr;
  a.act_scale = x_row_scale;  // per-row scales are linear in K: each partial carries them
  a.act_scale_const = x_row_scale ? 1.f : 1.f / h_scale;
  a.offsets = nullptr;
  a.n_rows = n_rows;
  a.n_experts = 1;
  a.out_rows = dim;
  a.rt_count = int(ceil_div(dim, kTmM));
  a.kc_count = int(ceil_div(inter, kChunkK));
  a.o_out = partials;
  a.o_row_map = nullptr;
  a.ldo = dim;
  a.round_o = 0;  // rounding belongs to the sum of the partials
  a.group_size = group_size > 0 ? group_size : 64;
  a.k_splits = std::max(1, k_splits);
  a.k_per = (a.kc_count + a.k_splits - 1) / a.k_splits;  // 128-row units take one chunk per stage
  if ((a.k_splits - 1) * a.k_per >= a.kc_count) return fail(DSM_ERR_INVALID_ARGUMENT, "expert_tm: empty K split");
  a.o_split_stride = n_rows * dim;
  return dispatch_tm<false>(wfmt, a, h_staged, rows_cap, as_stream(stream));
}

}  // namespace dsm
