// Grouped expert products at large token counts (prefill): tcgen05 MMA with TMEM
// accumulators, for fp8 128x128 block-scaled experts and f16-packed (bf16/fp32) experts --
// the shared expert among them.
//
// Work unit = (expert e, 128 weight rows, up to 256 staged rows of the expert). Persistent
// CTAs, warp-specialised:
//   warp 0      producer: per 64-wide K stage, bulk-copies the unit's fp8 codes (half of a
//               packed 128x128 tile, already in the layout the decode kernel reads) plus the
//               tile's fp32 block scale, and TMA-loads the 256 x 64 f16 activation box (128B
//               swizzle) from the staged rows, into a ring of load slots (as many as shared
//               memory holds: 3-4);
//   warp 1      MMA issuer (one elected thread): tcgen05.mma kind::f16, M=128, N = the
//               unit's rows rounded to 16 (up to 256), K=16 x 4 per stage, D in TMEM (two
//               buffers where they fit -- the down product -- so an epilogue overlaps the next
//               unit's main loop; the gate/up pair's two 256-column accumulators fill TMEM);
//               tcgen05.commit releases load slots and A slots and hands accumulators to the
//               epilogue;
//   warps 2-9   converters: e4m3 -> f16 (hardware cvt) times the block scale (f16 multiply),
//               written as the K-major SWIZZLE_128B f16 A operand into a two-slot ring of
//               its own, with bank-conflict-free 16-byte stores;
//   warps 10-21 epilogue: tcgen05.ld of the accumulators (warp w reads TMEM sub-partition
//               w % 4; the three warps of a sub-partition take alternate 16-column blocks),
//               activation row scale, SwiGLU (gate/up) or output rows (down).
// Shared memory bandwidth sets the pace: every stage moves the widened A tiles in and out,
// the activation rows in (TMA) and out (MMA) and the raw codes through the converters. The
// 256-row units read each A tile once per 256 rows instead of per 128 (4 KB of A + 8 KB of B
// per 128 tensor cycles of an N = 256 MMA).
//
// A and B of one kind::f16 MMA must share a type, and the bf16 activations rule out the fp8
// MMA kinds (fp8 activations would cost ~2% relative error), so the weights are widened to
// f16 in shared memory; the block scale is folded in there (one extra f16 rounding of the
// weight, 2^-11 relative) because it changes every 128 K and a TMEM accumulator cannot be
// rescaled between K blocks without reading it out.
#include <algorithm>
#include <mutex>

#include <type_traits>

#include "tcgen05.cuh"

namespace dsm {
namespace {

using namespace tc;

constexpr int kTcM = 128;            // weight rows per unit = one scale row block
constexpr int kTcK = 64;             // K per stage = one 128-byte swizzle row of f16
constexpr int kTcConvWarps = 8;
constexpr int kTcEpiWarps = 12;  // a multiple of 4: warps of one TMEM sub-partition share its columns
constexpr int kTcConvWarp0 = 2;
constexpr int kTcEpiWarp0 = kTcConvWarp0 + kTcConvWarps;  // 10
constexpr int kTcThreads = 32 * (kTcEpiWarp0 + kTcEpiWarps);
constexpr int kABytes = kTcM * kTcK * 2;
constexpr int kTcABufs = 2;     // widened A tiles: converted one stage ahead of the MMAs
constexpr int kTcMaxLoads = 8;  // load slots (sized at launch from the shared memory left)

// FMT: DSM_WFMT_FP8_B128 (codes widened and block-scaled by the converters) or DSM_WFMT_F16
// (f16 codes reshuffled into the swizzled layout; the per-expert prescale is undone in the
// epilogue). A load slot holds one 64-K stage: the BN activation rows (TMA, 128-byte swizzle)
// and the packed tile's codes for 64 K: slabs 2h, 2h+1 (fp8, 8 KB) or 4h .. 4h+3 (f16, 16 KB)
// of the 128-K tile, per matrix; the fp8 block scales go to a small side array. The widened
// A tiles live in their own two-slot ring, so the loads (whose latency sets the pace) keep
// more stages in flight than a ring of whole stages would.
// DUAL: the gate/up pair (matrices w1, w3 over the same row tile, SwiGLU epilogue). PAIR: the
// down product over two adjacent row tiles of one matrix, so each activation tile that lands
// in shared memory feeds two MMAs as it does for the gate/up pair.
template <int FMT, bool DUAL, bool PAIR = false>
struct TcCfg {
  static constexpr bool kFp8 = FMT == DSM_WFMT_FP8_B128;
  static constexpr int NM = (DUAL || PAIR) ? 2 : 1;
  static constexpr int BN = 256;
  static constexpr int kRawBytes = kFp8 ? 8192 : 16384;
  static constexpr int kMetaBytes = kFp8 ? 16 : 0;
  static constexpr int kBBytes = BN * kTcK * 2;
  static constexpr int kOffRaw = kBBytes;                         // load slot: [B][raw x NM]
  static constexpr int kLoadBytes = kBBytes + NM * kRawBytes;     // a multiple of 1024
  static constexpr int kABufBytes = NM * kABytes;
  static constexpr int kTxBytes = NM * (kRawBytes + kMetaBytes) + kBBytes;
  // accumulators double-buffered when two fit in the 512 TMEM columns
  static constexpr int kNBuf = 2 * NM * BN <= 512 ? 2 : 1;
  static constexpr int kTmemCols = kNBuf * NM * BN;
  static_assert(kLoadBytes % 1024 == 0, "load slots keep the 1024-byte alignment of the swizzled B tiles");
};

// shared memory past the A and load slots: barriers, block scales, TMEM slot, flags, unit prefix
constexpr size_t tc_tail_bytes(int n_experts) {
  return 8 * (2 * kTcMaxLoads + 2 * kTcABufs + 5) + 16 * 2 * kTcMaxLoads + 16 + size_t(n_experts + 1) * 4;
}

struct TcArgs {
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
  // single-matrix, unpaired product only: K ranges per (row tile, row chunk), each writing an
  // fp32 partial slab o_out + split * o_split_stride (rows [n_rows][ldo], staged-row order, no
  // row map or rounding); 0 or 1 = no split. k_per: 128-K chunks per range.
  int k_splits;
  int k_per;
  int64_t o_split_stride;
  // activation rows per TMA box (a multiple of 16, at most the unit width; 0 = the unit
  // width): a single group of few rows loads only the rows it has, not a 256-row box of
  // which the rows past the group are read for nothing
  int box_rows;
};

// Unit u's place: expert e, row tile rt, row chunk, K range ksp covering 64-K stages
// [ks0, ks1). K ranges sit between the row tiles and the row chunks.
struct TcUnit {
  int e, rt, chunk, ksp, ks0, ks1;
};

__device__ __forceinline__ int tc_group_first(const TcArgs& a, int e) { return a.offsets ? a.offsets[e] : 0; }
__device__ __forceinline__ int tc_group_count(const TcArgs& a, int e) {
  return a.offsets ? a.offsets[e + 1] - a.offsets[e] : int(a.n_rows);
}

__device__ __forceinline__ int tc_find_expert(const int* pre, int n_experts, int u) {
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

template <int FMT, bool DUAL, bool PAIR>
__global__ void __launch_bounds__(kTcThreads, 1) expert_tc_kernel(const TcArgs a,
                                                                  const __grid_constant__ CUtensorMap xmap,
                                                                  const int n_loads) {
  using C = TcCfg<FMT, DUAL, PAIR>;
  static_assert(!(DUAL && PAIR), "a unit is a gate/up pair or a pair of down row tiles");
  const int rtu = PAIR ? a.rt_count / 2 : a.rt_count;  // row-tile units per expert (rt_count even for PAIR)
  const int S = n_loads;  // load slots, 2 .. kTcMaxLoads
  constexpr int NM = C::NM, BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  // [A slots][load slots][block scales][barriers][TMEM slot, abort flag, unit prefix]
  uint8_t* abase = smem_raw + (base - raw0);
  uint8_t* lbase = abase + kTcABufs * C::kABufBytes;
  uint8_t* metas = lbase + size_t(S) * C::kLoadBytes;  // [slot][matrix] 16 bytes (bulk-copy aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(metas + 16 * 2 * kTcMaxLoads);
  uint64_t* empty = full + kTcMaxLoads;
  uint64_t* conv = empty + kTcMaxLoads;
  uint64_t* aempty = conv + kTcABufs;
  uint64_t* tfull = aempty + kTcABufs;
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
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kTcABufs; ++b) {
      mbar_init(&conv[b], kTcConvWarps);
      mbar_init(&aempty[b], 1);
    }
    for (int b = 0; b < C::kNBuf; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kTcEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {  // TMEM: the accumulator buffers
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp == 0) {  // units per expert: rt_count x ceil(count / BN)
    int carry = 0;
    if (lane == 0) pre[0] = 0;
    for (int b0 = 0; b0 < E; b0 += 32) {
      const int e = b0 + lane;
      int v = 0;
      if (e < E) {
        const int cnt = tc_group_count(a, e);
        v = cnt > 0 ? rtu * ((cnt + BN - 1) / BN) * (a.k_splits > 1 ? a.k_splits : 1) : 0;
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
  const int tile_b = tile_bytes(FMT, 0);
  const uint8_t* tiles[2] = {a.wa + hdr_bytes, DUAL ? a.wb + hdr_bytes : a.wa + hdr_bytes};
  const int nks = 2 * a.kc_count;  // 64-wide K stages per unsplit unit
  const int nsp = a.k_splits > 1 ? a.k_splits : 1;
  auto unit = [&](int u) {
    TcUnit w;
    w.e = tc_find_expert(pre, E, u);
    const int nch = (tc_group_count(a, w.e) + BN - 1) / BN;
    const int local = u - pre[w.e];
    w.rt = local / (nch * nsp);
    const int r2 = local % (nch * nsp);
    w.chunk = r2 % nch;
    w.ksp = r2 / nch;
    w.ks0 = nsp > 1 ? 2 * w.ksp * a.k_per : 0;
    w.ks1 = nsp > 1 ? min(nks, w.ks0 + 2 * a.k_per) : nks;
    return w;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    const int box = a.box_rows > 0 ? a.box_rows : BN;
    const uint32_t tx_bytes = uint32_t(C::kTxBytes - C::kBBytes + box * kTcK * 2);
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const TcUnit w = unit(u);
        const int e = w.e, rt = w.rt;
        const int row0 = tc_group_first(a, e) + w.chunk * BN;
        // first row tile of the unit: rt (gate/up pair, both matrices) or 2 rt, 2 rt + 1 (PAIR)
        const int64_t tile0 = (int64_t(e) * a.rt_count + (PAIR ? 2 * rt : rt)) * a.kc_count;
        for (int ks = w.ks0; ks < w.ks1; ++ks) {
          if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* st = lbase + size_t(s) * C::kLoadBytes;
          const int kc = ks >> 1, half = ks & 1;
          mbar_arrive_expect_tx(&full[s], tx_bytes);
#pragma unroll
          for (int m = 0; m < NM; ++m) {
            const uint8_t* tile = tiles[m] + (tile0 + (PAIR ? m * a.kc_count : 0) + kc) * tile_b;
            bulk_g2s(st + C::kOffRaw + m * C::kRawBytes, tile + half * C::kRawBytes, C::kRawBytes, &full[s], pol_w);
            if (C::kFp8) bulk_g2s(metas + (s * NM + m) * 16, tile + 16384, 16, &full[s], pol_w);
          }
          tma_load_3d(smem_u32(st), &xmap, half * kTcK, row0, kc, &full[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok)
        for (int i = 0; i < 100; ++i) __nanosleep(1000);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0, ab = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      int j = 0;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++j) {
        const TcUnit w = unit(u);
        const int rows = min(BN, tc_group_count(a, w.e) - w.chunk * BN);
        const int n_mma = min(BN, (rows + 15) / 16 * 16);
        const uint32_t idesc = umma_idesc_f16(kTcM, n_mma);
        const int buf = j % C::kNBuf;
        if (*abort_flag || !mbar_wait(&tempty[buf], ((j / C::kNBuf) & 1) ^ 1u)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        for (int ks = w.ks0; ks < w.ks1; ++ks) {
          if (*abort_flag || !mbar_wait(&conv[ab], aph) || !mbar_wait(&full[s], ph)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sb = smem_u32(lbase + size_t(s) * C::kLoadBytes);
          const uint32_t sa = smem_u32(abase + ab * C::kABufBytes);
#pragma unroll
          for (int kk = 0; kk < kTcK / 16; ++kk) {
            const uint64_t bdesc = umma_desc_sw128(sb) + uint64_t(kk * 2);
#pragma unroll
            for (int m = 0; m < NM; ++m) {
              const uint64_t adesc = umma_desc_sw128(sa + m * kABytes) + uint64_t(kk * 2);
              const uint32_t d = tmem + uint32_t((buf * NM + m) * BN);
              umma_f16(d, adesc, bdesc, idesc, (ks > w.ks0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty[s]);    // load slot free once these MMAs have read B (the
          umma_commit(&aempty[ab]);  // converters were done with its codes before) and A
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
          if (++ab == kTcABufs) {
            ab = 0;
            aph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);  // accumulator ready for the epilogue
      }
      // all MMAs issued by this thread complete before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp < kTcEpiWarp0) {
    // ------------------------------------------------------------------ converters
    const int cw = warp - kTcConvWarp0;  // 0..7
    const int g = lane >> 2, q = lane & 3;
    int s = 0, ab = 0;
    uint32_t ph = 0, aph = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      bool ok = true;
      const TcUnit w = unit(u);
      for (int ks = w.ks0; ks < w.ks1; ++ks) {
        // the stage's codes have landed, and the MMAs two stages back have released A slot ab
        if (*abort_flag || !mbar_wait(&full[s], ph) || !mbar_wait(&aempty[ab], aph ^ 1u)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        uint8_t* st = lbase + size_t(s) * C::kLoadBytes;
#pragma unroll
        for (int m = 0; m < NM; ++m) {
          const uint32_t rawm = smem_u32(st + C::kOffRaw + m * C::kRawBytes);
          const uint32_t am = smem_u32(abase + ab * C::kABufBytes + m * kABytes);
          if constexpr (!C::kFp8) {
            // f16 codes: 4 k16 slabs x 8 m16 tiles of 512 B; lane holds rows r0, r0+8 at k 4q..4q+3
#pragma unroll
            for (int bi = 0; bi < 4; ++bi) {
              const int blk = cw + 8 * bi;
              const int sl = blk >> 3, mt = blk & 7;
              const uint4 v = lds128(rawm + (blk * 32 + lane) * 16);
              const int r0 = mt * 16 + g, r1 = r0 + 8;
              const int k = sl * 16 + q * 4;
              const int ch = k >> 3, sub = (k & 7) * 2;
              const uint32_t p0 = am + r0 * 128 + ((ch ^ (r0 & 7)) << 4) + sub;
              const uint32_t p1 = am + r1 * 128 + ((ch ^ (r1 & 7)) << 4) + sub;
              asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(p0), "r"(v.x), "r"(v.y) : "memory");
              asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(p1), "r"(v.z), "r"(v.w) : "memory");
            }
            continue;
          }
          const float sc = *reinterpret_cast<const float*>(metas + (s * NM + m) * 16);
          const __half2 s2 = __float2half2_rn(sc);
          const uint32_t sbits = *reinterpret_cast<const uint32_t*>(&s2);
          // 16 blocks of 512 B (2 slabs x 8 m16 tiles); warp cw converts blocks cw (slab 0) and
          // cw + 8 (slab 1): lane (g, q) holds rows r0 = 16 cw + g and r0 + 8 at k 8q..8q+7 of each
          // slab, i.e. 16-byte chunk q of slab 0 and chunk 4 + q of slab 1 in the swizzled rows.
          // A 16-byte store serves 8 lanes per pass (g = 2p, 2p + 1); lanes of odd g store the
          // slab-1 chunk first, so the pass covers chunks {q ^ g} and {(4 + q) ^ g'}: all eight
          // 16-byte bank groups, no conflict.
          uint32_t h[2][8];
#pragma unroll
          for (int bi = 0; bi < 2; ++bi) {
            const uint4 v = lds128(rawm + ((cw + 8 * bi) * 32 + lane) * 16);
            e4m3x4_to_f16(v.x, h[bi][0], h[bi][1]);  // row r0, k 8q..8q+3
            e4m3x4_to_f16(v.y, h[bi][2], h[bi][3]);  // row r0, k 8q+4..8q+7
            e4m3x4_to_f16(v.z, h[bi][4], h[bi][5]);  // row r0+8
            e4m3x4_to_f16(v.w, h[bi][6], h[bi][7]);
#pragma unroll
            for (int i = 0; i < 8; ++i) h[bi][i] = hmul2_bits(h[bi][i], sbits);
          }
          const int odd = g & 1;
          const int r0 = cw * 16 + g;
          const uint32_t row0 = am + r0 * 128, row1 = row0 + 8 * 128;
#pragma unroll
          for (int o = 0; o < 2; ++o) {
            const int bi = o ^ odd;  // slab this lane stores in pass o
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = bi ? h[1][i] : h[0][i];
            const uint32_t cx = uint32_t(((bi * 4 + q) ^ g) << 4);  // r0 & 7 == r1 & 7 == g
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(row0 + cx), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                         "r"(w[3])
                         : "memory");
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(row1 + cx), "r"(w[4]), "r"(w[5]), "r"(w[6]),
                         "r"(w[7])
                         : "memory");
          }
        }
        fence_async_smem();  // generic-proxy writes -> visible to the tensor core's async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[ab]);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
        if (++ab == kTcABufs) {
          ab = 0;
          aph ^= 1u;
        }
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int sp = warp & 3;  // TMEM sub-partition of this warp: lanes 32*sp .. 32*sp+31
    const int eh = (warp - kTcEpiWarp0) >> 2;  // which of the sub-partition's column blocks
    const int rloc = 32 * sp + lane;
    int j = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++j) {
      const TcUnit w = unit(u);
      const int e = w.e, rt = w.rt, chunk = w.chunk;
      const int off = tc_group_first(a, e);
      const int rows = min(BN, tc_group_count(a, e) - chunk * BN);
      const int buf = j % C::kNBuf;
      if (*abort_flag || !mbar_wait_backoff(&tfull[buf], (j / C::kNBuf) & 1, 200)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const float wmul_a = reinterpret_cast<const float*>(a.wa)[e];
      const float wmul_b = DUAL ? reinterpret_cast<const float*>(a.wb)[e] : wmul_a;
      const uint32_t lane_base = tmem + (uint32_t(32 * sp) << 16);
      for (int cb = 16 * eh; cb < rows; cb += 16 * (kTcEpiWarps / 4)) {
        uint32_t gv[16], uv[16];
        tmem_ld16(lane_base + uint32_t(buf * NM * BN + cb), gv);
        if (NM == 2) tmem_ld16(lane_base + uint32_t((buf * NM + 1) * BN + cb), uv);
        tmem_ld_wait();
        // all 16 columns are computed without a branch (columns past `rows` hold unused
        // accumulators) so their chains interleave, and only the stores are guarded; the
        // block's 16 row scales come in one guarded load per lane, broadcast with a constant
        // source lane per column
        const int cl = cb + (lane & 15);
        const int rl = off + chunk * BN + cl;
        const float xs_b = (cl < rows && a.act_scale) ? a.act_scale[rl] : a.act_scale_const;
        if constexpr (DUAL) {
          const bool rg = a.round_gu & 1, rh = a.round_gu & 2;
          __half* hp = a.h_out + (int64_t(rt) * a.h_rows_cap + off + chunk * BN + cb) * kStagePitch + rloc;
          auto block = [&](auto silu_tag) {
#pragma unroll
            for (int i0 = 0; i0 < 16; i0 += 8) {
              float hv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float xs = __shfl_sync(0xffffffffu, xs_b, i0 + i);
                float gg = __uint_as_float(gv[i0 + i]) * xs * wmul_a;
                float uu = __uint_as_float(uv[i0 + i]) * xs * wmul_b;
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
#pragma unroll
          for (int m = 0; m < NM; ++m) {
            const int d = (rt * NM + m) * kTcM + rloc;  // output feature: row of row tile rt * NM + m
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float xs = __shfl_sync(0xffffffffu, xs_b, i);
              const int orow = __shfl_sync(0xffffffffu, or_b, i);
              float v = __uint_as_float(m ? uv[i] : gv[i]) * xs * wmul_a;
              if (nsp > 1) {  // a partial of the K range, in staged-row order: the split sum rounds
                if (cb + i < rows && d < a.out_rows)
                  a.o_out[int64_t(w.ksp) * a.o_split_stride + int64_t(off + chunk * BN + cb + i) * a.ldo + d] = v;
                continue;
              }
              v = a.round_o ? bf16_round(v) : v;
              if (cb + i < rows && d < a.out_rows) a.o_out[int64_t(orow) * a.ldo + d] = v;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
  }
}

template <int FMT, bool DUAL, bool PAIR = false>
int launch_tc(TcArgs a, const void* staged, int64_t rows_cap, cudaStream_t stream) {
  using C = TcCfg<FMT, DUAL, PAIR>;
  // one group of rows (offsets NULL): the box covers its rows only (whole units of 256 rows
  // above that). Grouped calls keep the unit width: their counts are on the device.
  a.box_rows = a.offsets ? 0 : int(std::min<int64_t>(C::BN, (a.n_rows + 15) / 16 * 16));
  CUtensorMap map;
  if (int rc = make_stage_map(&map, staged, rows_cap, a.kc_count, a.box_rows > 0 ? a.box_rows : C::BN)) return rc;
  int dev = 0, optin = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return check_launch("expert_tc device attribute");
  // as many load slots as the shared memory left by the A slots holds
  const size_t fixed = 1024 + size_t(kTcABufs) * C::kABufBytes + tc_tail_bytes(a.n_experts);
  const int n_loads = size_t(optin) > fixed ? int(std::min<size_t>(kTcMaxLoads, (size_t(optin) - fixed) / C::kLoadBytes)) : 0;
  if (n_loads < 2) return fail(DSM_ERR_UNSUPPORTED, "expert_tc: too many experts for the shared-memory ring");
  const size_t smem = fixed + size_t(n_loads) * C::kLoadBytes;
  auto kern = expert_tc_kernel<FMT, DUAL, PAIR>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return check_launch("expert_tc smem attribute");
  kern<<<persistent_ctas(), kTcThreads, smem, stream>>>(a, map, n_loads);
  return check_launch("expert_tc");
}

}  // namespace

// ---- host side ------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_stage_map(CUtensorMap* map, const void* staged, int64_t rows_cap, int k_chunks, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return fail(DSM_ERR_CUDA, "expert_tc: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {cuuint64_t(kStagePitch), cuuint64_t(rows_cap), cuuint64_t(k_chunks)};
  const cuuint64_t strides[2] = {cuuint64_t(kStagePitch) * 2, cuuint64_t(rows_cap) * kStagePitch * 2};
  const cuuint32_t box[3] = {cuuint32_t(kTcK), cuuint32_t(box_rows), 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(staged), dims, strides, box, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSM_ERR_CUDA, "expert_tc: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return DSM_OK;
}

// Entry points used by the expert dispatch (expert.cu) for the fp8 large-token regime.
bool tc_supports(int wfmt) { return wfmt == DSM_WFMT_FP8_B128 || wfmt == DSM_WFMT_F16; }

int expert_tc_gate_up(int wfmt, const void* x_staged, const float* x_row_scale, int64_t rows_cap, int dim,
                      const int32_t* offsets, int n_experts, const void* w1, const void* w3, int inter, int act,
                      float limit, int round_gu, void* h_staged, float h_scale, int64_t n_rows, void* stream) {
  TcArgs a{};
  a.wa = static_cast<const uint8_t*>(w1);
  a.wb = static_cast<const uint8_t*>(w3);
  a.act_scale = x_row_scale;
  a.act_scale_const = 1.f;
  a.offsets = offsets;
  a.n_rows = n_rows;
  a.n_experts = n_experts;
  a.out_rows = inter;
  a.rt_count = int(ceil_div(inter, kTcM));
  a.kc_count = int(ceil_div(dim, kChunkK));
  a.act = act;
  a.limit = limit;
  a.round_gu = round_gu;
  a.h_scale = h_scale;
  a.h_out = static_cast<__half*>(h_staged);
  a.h_rows_cap = rows_cap;
  if (wfmt == DSM_WFMT_F16) return launch_tc<DSM_WFMT_F16, true>(a, x_staged, rows_cap, as_stream(stream));
  return launch_tc<DSM_WFMT_FP8_B128, true>(a, x_staged, rows_cap, as_stream(stream));
}

int expert_tc_down(int wfmt, const void* h_staged, float h_scale, int64_t rows_cap, int inter, const int32_t* offsets,
                   int n_experts, const void* w2, int dim, int round_o, float* o_rows, int ldo,
                   const int32_t* o_row_map, int64_t n_rows, void* stream, const float* x_row_scale) {
  TcArgs a{};
  a.wa = static_cast<const uint8_t*>(w2);
  a.wb = nullptr;
  a.act_scale = x_row_scale;
  a.act_scale_const = x_row_scale ? 1.f : 1.f / h_scale;
  a.offsets = offsets;
  a.n_rows = n_rows;
  a.n_experts = n_experts;
  a.out_rows = dim;
  a.rt_count = int(ceil_div(dim, kTcM));
  a.kc_count = int(ceil_div(inter, kChunkK));
  a.o_out = o_rows;
  a.o_row_map = o_row_map;
  a.ldo = ldo;
  a.round_o = round_o;
  if (wfmt == DSM_WFMT_F16) return launch_tc<DSM_WFMT_F16, false>(a, h_staged, rows_cap, as_stream(stream));
  // fp8 with an even number of output row tiles: two per unit (measured on the 16,384-token
  // call: 2.72 -> 2.56 ms). The f16 tiles are twice the bytes, so paired units would leave
  // two load slots, and the shared expert's down product measured slower that way.
  if (a.rt_count % 2 == 0) return launch_tc<DSM_WFMT_FP8_B128, false, true>(a, h_staged, rows_cap, as_stream(stream));
  return launch_tc<DSM_WFMT_FP8_B128, false>(a, h_staged, rows_cap, as_stream(stream));
}

int expert_tc_split(int wfmt, const void* x_staged, const float* x_row_scale, int64_t rows_cap, int k_dim,
                    const int32_t* offsets, int n_groups, const void* w_packed, int out_dim, int64_t n_rows,
                    int k_splits, int k_per, float* parts, void* stream) {
  TcArgs a{};
  a.wa = static_cast<const uint8_t*>(w_packed);
  a.wb = nullptr;
  a.act_scale = x_row_scale;
  a.act_scale_const = 1.f;
  a.offsets = offsets;
  a.n_rows = n_rows;
  a.n_experts = n_groups;
  a.out_rows = out_dim;
  a.rt_count = int(ceil_div(out_dim, kTcM));
  a.kc_count = int(ceil_div(k_dim, kChunkK));
  a.o_out = parts;
  a.o_row_map = nullptr;
  a.ldo = out_dim;
  a.round_o = 0;
  a.k_splits = k_splits;
  a.k_per = k_per;
  a.o_split_stride = n_rows * int64_t(out_dim);
  if (wfmt == DSM_WFMT_F16) return launch_tc<DSM_WFMT_F16, false>(a, x_staged, rows_cap, as_stream(stream));
  return launch_tc<DSM_WFMT_FP8_B128, false>(a, x_staged, rows_cap, as_stream(stream));
}

}  // namespace dsm
