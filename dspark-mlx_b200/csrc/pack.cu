// Load-time weight preparation.
//
// dsm_pack_weights turns stacked expert weights in the reference layout ([E, out, in],
// nn.Linear convention, dspark_mlx/loading.py:88-100 / model/moe.py:118-120) into the tile
// stream the expert kernels read with one bulk copy per pipeline stage:
//
//   header   float[E] per-expert multiplier (F16 and affine: the inverse of a power-of-two
//            prescale; FP4: per-tensor scale; FP8: 1), padded to a multiple of 256 bytes
//   tiles    for e, for row tile rt (128 rows), for K chunk kc (128 columns):
//              codes  format dependent, below
//              meta   per-tile scales (format dependent)
//
// F16, FP8 codes (the weight-streaming kernel): [slab][m16 tile 0..7][lane 0..31][16 bytes]
// -- one ld.shared.v4 per lane per m16 tile per slab, already in mma.m16n8k16 A-fragment
// order. Lane (g = lane/4, q = lane%4) of m16 tile m holds rows r0 = 16m+g and r1 = r0+8;
// its 16 bytes are [row r0 part][row r1 part] where the part covers K columns
//   F16 (slab = 16 K): 4q .. 4q+3 (4 f16);  FP8 (slab = 32 K): 8q .. 8q+7 (8 bytes).
// The kernel multiplies these against activations loaded with the same K subset per lane,
// which is a consistent permutation of K inside each MMA and leaves the dot product
// unchanged.
// FP4, AFF8, AFF4 codes (the tensor-memory kernel): row-sliced, [16-byte chunk c][row
// 0..127][16 bytes], so that one converter thread per row reads a chunk with one
// ld.shared.v4 and a warp reads 512 contiguous bytes:
//   FP4  chunk = 32 K: byte j = K 32c+2j (low nibble), 32c+2j+1 (high nibble)
//   AFF8 chunk = 16 K: byte j = K 16c+j
//   AFF4 chunk = 32 K: word w holds K 32c+8w .. +7 in nibble order k0,k2,k4,k6,k1,k3,k5,k7
//        (nibble i and i+4 of a word are one K pair, for the magic-number unpack)
// Affine meta: per row and group, the f16 pair (scale, bias) times the expert's prescale
// 2^p (max |w| * 2^p in [2^14, 2^15); the header holds 2^-p), so a converter forms
// w * 2^p = q * scale' + bias' with one f16 fma.
//
// dsm_affine_quantize restates MLX's affine quantize (called by MoE.quantize,
// dspark_mlx/model/moe.py:124-130): per group, an fp32 scale/bias with the edge of larger
// magnitude snapped so that zero is exact, q = clip(rint((w - bias) / scale), 0, 2^bits-1),
// scales and biases stored in the weight dtype.
#include <algorithm>

#include "common.cuh"

namespace dsm {
namespace {

__global__ void fill_header_kernel(float* header, int n, float v) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) header[i] = v;
}

template <typename T>
__device__ __forceinline__ float src_at(const void* p, int64_t i) {
  return load_as_float(static_cast<const T*>(p), i);
}

template <typename T>
__global__ void expert_amax_kernel(const T* __restrict__ w, int64_t per_expert, float* __restrict__ amax) {
  const int e = blockIdx.y;
  float m = 0.f;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < per_expert; i += int64_t(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(load_as_float(w + int64_t(e) * per_expert, i)));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(amax + e), __float_as_int(m));
}

// max |w| over an expert's affine groups: |w| <= max(|bias|, |bias + qmax * scale|)
__global__ void affine_amax_kernel(const __nv_bfloat16* __restrict__ scales, const __nv_bfloat16* __restrict__ biases,
                                   int64_t groups_per_expert, float qmax, float* __restrict__ amax) {
  const int e = blockIdx.y;
  float m = 0.f;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < groups_per_expert;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t j = int64_t(e) * groups_per_expert + i;
    const float s = __bfloat162float(scales[j]), b = __bfloat162float(biases[j]);
    m = fmaxf(m, fmaxf(fabsf(b), fabsf(fmaf(qmax, s, b))));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(amax + e), __float_as_int(m));
}

__device__ __forceinline__ int prescale_exp(float amax) {
  if (!(amax > 0.f) || !isfinite(amax)) return 0;
  int ex;
  frexpf(amax, &ex);
  const int s = 15 - ex;
  return s < -100 ? -100 : (s > 100 ? 100 : s);
}

__global__ void finalize_prescale_header_kernel(float* header, int n_experts) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e < n_experts) header[e] = ldexpf(1.f, -prescale_exp(header[e]));
}

struct PackArgs {
  int wfmt, n_experts, rows, cols, group_size, rt_count, kc_count;
  const void* codes;
  const void* scales;
  const void* biases;
  const float* header;  // F16: per-expert amax (read-only here)
  uint8_t* tiles;
  int src_dtype;
};

// One block per tile; threads loop over the tile's 16-byte lane chunks, then its metadata.
__global__ void __launch_bounds__(256) pack_tiles_kernel(PackArgs a) {
  const int64_t tile = blockIdx.x;
  const int kc = int(tile % a.kc_count);
  const int rt = int((tile / a.kc_count) % a.rt_count);
  const int e = int(tile / (int64_t(a.kc_count) * a.rt_count));
  const int code_bytes = tile_code_bytes(a.wfmt);
  uint8_t* dst = a.tiles + tile * int64_t(tile_bytes(a.wfmt, a.group_size));
  const int slab_k = a.wfmt == DSM_WFMT_F16 ? 16 : 32;  // F16 / FP8 (fragment order)
  const int n_chunks = code_bytes / 16;
  const int64_t R = a.rows, K = a.cols;
  float up = 1.f;
  const bool affine = a.wfmt == DSM_WFMT_AFFINE8 || a.wfmt == DSM_WFMT_AFFINE4;
  if (a.wfmt == DSM_WFMT_F16 || affine) up = ldexpf(1.f, prescale_exp(a.header[e]));
  if (a.wfmt == DSM_WFMT_FP4_G32) {  // row-sliced: [chunk][row][16 bytes]
    const uint8_t* src = static_cast<const uint8_t*>(a.codes);
    const int64_t kbytes = K / 2;
    for (int c = threadIdx.x; c < n_chunks; c += blockDim.x) {
      const int cc = c >> 7, rr = c & 127;
      const int64_t r = int64_t(rt) * kTileRows + rr;
      const int64_t kb0 = (int64_t(kc) * kChunkK + 32 * cc) / 2;
      uint8_t out[16];
      for (int j = 0; j < 16; ++j)
        out[j] = (r < R && kb0 + j < kbytes) ? src[(int64_t(e) * R + r) * kbytes + kb0 + j] : uint8_t(0);
      uint4 v;
      memcpy(&v, out, 16);
      *reinterpret_cast<uint4*>(dst + 16 * c) = v;
    }
  }
  if (affine) {  // row-sliced, 8-bit: 16 K per chunk; 4-bit: 32 K per chunk
    const uint8_t* src = static_cast<const uint8_t*>(a.codes);
    const bool b8 = a.wfmt == DSM_WFMT_AFFINE8;
    const int64_t kbytes = b8 ? K : K / 2;
    for (int c = threadIdx.x; c < n_chunks; c += blockDim.x) {
      const int cc = c >> 7, rr = c & 127;
      const int64_t r = int64_t(rt) * kTileRows + rr;
      const int64_t k0 = int64_t(kc) * kChunkK + (b8 ? 16 : 32) * cc;
      uint8_t out[16];
      if (b8) {
        for (int j = 0; j < 16; ++j)
          out[j] = (r < R && k0 + j < K) ? src[(int64_t(e) * R + r) * kbytes + k0 + j] : uint8_t(0);
      } else {
        for (int w = 0; w < 4; ++w) {
          uint8_t nib[8];
          for (int i = 0; i < 8; ++i) {
            const int64_t k = k0 + 8 * w + i;
            uint8_t v = 0;
            if (r < R && k < K) {
              const uint8_t b = src[(int64_t(e) * R + r) * kbytes + k / 2];
              v = (k & 1) ? (b >> 4) : (b & 0xF);
            }
            nib[i] = v;
          }
          const uint8_t order[8] = {nib[0], nib[2], nib[4], nib[6], nib[1], nib[3], nib[5], nib[7]};
          for (int j = 0; j < 4; ++j) out[4 * w + j] = uint8_t(order[2 * j] | (order[2 * j + 1] << 4));
        }
      }
      uint4 v;
      memcpy(&v, out, 16);
      *reinterpret_cast<uint4*>(dst + 16 * c) = v;
    }
  }
  for (int c = threadIdx.x; c < n_chunks && (a.wfmt == DSM_WFMT_F16 || a.wfmt == DSM_WFMT_FP8_B128);
       c += blockDim.x) {
    const int lane = c & 31, m = (c >> 5) & 7, slab = c >> 8;
    const int g = lane >> 2, q = lane & 3;
    const int64_t kb = int64_t(kc) * kChunkK + int64_t(slab) * slab_k;
    uint8_t out[16];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int64_t r = int64_t(rt) * kTileRows + 16 * m + g + 8 * half;
      uint8_t* o = out + 8 * half;
      const bool row_ok = r < R;
      if (a.wfmt == DSM_WFMT_F16) {
        for (int j = 0; j < 4; ++j) {
          const int64_t k = kb + 4 * q + j;
          float v = 0.f;
          if (row_ok && k < K) {
            const int64_t i = (int64_t(e) * R + r) * K + k;
            v = (a.src_dtype == DSM_DT_BF16 ? src_at<__nv_bfloat16>(a.codes, i) : src_at<float>(a.codes, i)) * up;
          }
          const __half h = __float2half_rn(v);
          const uint16_t bits = *reinterpret_cast<const uint16_t*>(&h);
          o[2 * j] = uint8_t(bits & 0xFF);
          o[2 * j + 1] = uint8_t(bits >> 8);
        }
      } else {  // FP8
        const uint8_t* src = static_cast<const uint8_t*>(a.codes);
        for (int j = 0; j < 8; ++j) {
          const int64_t k = kb + 8 * q + j;
          o[j] = (row_ok && k < K) ? src[(int64_t(e) * R + r) * K + k] : uint8_t(0);
        }
      }
    }
    uint4 v;
    memcpy(&v, out, 16);
    *reinterpret_cast<uint4*>(dst + 16 * c) = v;
  }
  // metadata
  uint8_t* meta = dst + code_bytes;
  if (a.wfmt == DSM_WFMT_FP8_B128) {
    if (threadIdx.x < 4) {
      float v = 0.f;
      if (threadIdx.x == 0) {
        const int64_t sr = ceil_div(R, 128), sc = ceil_div(K, 128);
        v = static_cast<const float*>(a.scales)[(int64_t(e) * sr + rt) * sc + kc];
      }
      reinterpret_cast<float*>(meta)[threadIdx.x] = v;
    }
  } else if (a.wfmt == DSM_WFMT_FP4_G32) {
    const uint8_t* gs = static_cast<const uint8_t*>(a.scales);
    const int64_t groups = K / 32;
    for (int i = threadIdx.x; i < kTileRows * 4; i += blockDim.x) {
      const int rr = i >> 2, gg = i & 3;
      const int64_t r = int64_t(rt) * kTileRows + rr;
      const int64_t grp = int64_t(kc) * 4 + gg;
      meta[i] = (r < R && grp < groups) ? gs[(int64_t(e) * R + r) * groups + grp] : uint8_t(0);
    }
  } else if (affine) {
    const int gpt = kChunkK / a.group_size;  // groups per tile row
    const int64_t groups = K / a.group_size;
    const __nv_bfloat16* sc = static_cast<const __nv_bfloat16*>(a.scales);
    const __nv_bfloat16* bi = static_cast<const __nv_bfloat16*>(a.biases);
    __half* m16 = reinterpret_cast<__half*>(meta);
    for (int i = threadIdx.x; i < kTileRows * gpt; i += blockDim.x) {
      const int rr = i / gpt, gg = i % gpt;
      const int64_t r = int64_t(rt) * kTileRows + rr;
      const int64_t grp = int64_t(kc) * gpt + gg;
      const bool ok = r < R && grp < groups;
      const int64_t j = (int64_t(e) * R + r) * groups + grp;
      // bf16 times a power of two: exact in f16 within its normal range
      m16[2 * i] = __float2half_rn(ok ? __bfloat162float(sc[j]) * up : 0.f);
      m16[2 * i + 1] = __float2half_rn(ok ? __bfloat162float(bi[j]) * up : 0.f);
    }
  }
}

template <typename T>
__global__ void affine_quantize_kernel(const T* __restrict__ w, int64_t n_rows, int cols, int gs, int bits,
                                       uint8_t* __restrict__ codes, T* __restrict__ scales, T* __restrict__ biases) {
  const int groups = cols / gs;
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= n_rows * groups) return;
  const int64_t row = gid / groups;
  const int grp = int(gid % groups);
  const T* src = w + row * cols + int64_t(grp) * gs;
  float wmax = -INFINITY, wmin = INFINITY;
  for (int i = 0; i < gs; ++i) {
    const float v = load_as_float(src, i);
    wmax = fmaxf(wmax, v);
    wmin = fminf(wmin, v);
  }
  const float n_bins = float((1 << bits) - 1);
  const bool mask = fabsf(wmin) > fabsf(wmax);
  float scale = fmaxf((wmax - wmin) / n_bins, 1e-7f);
  scale = mask ? scale : -scale;
  const float edge = mask ? wmin : wmax;
  const float q0 = rintf(edge / scale);
  if (q0 != 0.f) scale = edge / q0;
  const float bias = q0 == 0.f ? 0.f : edge;
  uint8_t* dst = codes + row * (int64_t(cols) * bits / 8) + int64_t(grp) * gs * bits / 8;
  for (int i = 0; i < gs; i += (bits == 8 ? 1 : 2)) {
    const float q_a = fminf(fmaxf(rintf((load_as_float(src, i) - bias) / scale), 0.f), n_bins);
    if (bits == 8) {
      dst[i] = uint8_t(q_a);
    } else {
      const float q_b = fminf(fmaxf(rintf((load_as_float(src, i + 1) - bias) / scale), 0.f), n_bins);
      dst[i / 2] = uint8_t(uint32_t(q_a) | (uint32_t(q_b) << 4));
    }
  }
  if constexpr (sizeof(T) == 2) {
    scales[gid] = __float2bfloat16_rn(scale);
    biases[gid] = __float2bfloat16_rn(bias);
  } else {
    scales[gid] = scale;
    biases[gid] = bias;
  }
}

}  // namespace
}  // namespace dsm

extern "C" size_t dsm_packed_bytes(int wfmt, int n_experts, int rows, int cols, int group_size) {
  using namespace dsm;
  if (wfmt < DSM_WFMT_F16 || wfmt > DSM_WFMT_AFFINE4 || n_experts <= 0 || rows <= 0 || cols <= 0) return 0;
  const int64_t tiles = int64_t(n_experts) * ceil_div(rows, kTileRows) * ceil_div(cols, kChunkK);
  return size_t(packed_header_bytes(n_experts) + tiles * tile_bytes(wfmt, group_size));
}

extern "C" int dsm_pack_weights(int wfmt, int n_experts, int rows, int cols, int group_size, int src_dtype,
                                const void* codes, const void* scales, const void* biases, const float* tensor_scale,
                                void* packed, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(wfmt >= DSM_WFMT_F16 && wfmt <= DSM_WFMT_AFFINE4, "dsm_pack_weights: unknown format");
  DSM_REQUIRE(n_experts > 0 && rows > 0 && cols > 0, "dsm_pack_weights: bad shape");
  DSM_REQUIRE(codes && packed, "dsm_pack_weights: NULL pointer");
  DSM_REQUIRE((reinterpret_cast<uintptr_t>(packed) & 255) == 0, "dsm_pack_weights: packed must be 256-byte aligned");
  if (wfmt == DSM_WFMT_F16)
    DSM_REQUIRE(src_dtype == DSM_DT_F32 || src_dtype == DSM_DT_BF16, "dsm_pack_weights: F16 source must be F32 or BF16");
  if (wfmt == DSM_WFMT_FP8_B128) DSM_REQUIRE(scales, "dsm_pack_weights: FP8 needs block scales");
  if (wfmt == DSM_WFMT_FP4_G32) {
    DSM_REQUIRE(scales && tensor_scale, "dsm_pack_weights: FP4 needs group and tensor scales");
    DSM_REQUIRE(cols % 32 == 0, "dsm_pack_weights: FP4 needs cols % 32 == 0");
  }
  if (wfmt == DSM_WFMT_AFFINE8 || wfmt == DSM_WFMT_AFFINE4) {
    DSM_REQUIRE(scales && biases, "dsm_pack_weights: affine needs scales and biases");
    const bool gs_ok = wfmt == DSM_WFMT_AFFINE8 ? (group_size == 32 || group_size == 64 || group_size == 128)
                                                 : (group_size == 64 || group_size == 128);
    DSM_REQUIRE(gs_ok, "dsm_pack_weights: affine group_size must be 32/64/128 (8-bit) or 64/128 (4-bit)");
    DSM_REQUIRE(cols % group_size == 0, "dsm_pack_weights: cols must be a multiple of group_size");
    DSM_REQUIRE(src_dtype == DSM_DT_BF16, "dsm_pack_weights: affine scales/biases must be BF16");
  }
  if (wfmt == DSM_WFMT_AFFINE4) DSM_REQUIRE(cols % 2 == 0, "dsm_pack_weights: 4-bit needs even cols");
  cudaStream_t s = as_stream(stream);
  float* header = static_cast<float*>(packed);
  const int64_t per_expert = int64_t(rows) * cols;
  if (wfmt == DSM_WFMT_F16) {
    if (cudaMemsetAsync(header, 0, sizeof(float) * n_experts, s) != cudaSuccess) return check_launch("memset");
    dim3 grid(unsigned(std::min<int64_t>(ceil_div(per_expert, 256), 1024)), unsigned(n_experts));
    if (src_dtype == DSM_DT_BF16)
      expert_amax_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(codes), per_expert, header);
    else
      expert_amax_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(codes), per_expert, header);
    if (int rc = check_launch("expert_amax")) return rc;
  } else if (wfmt == DSM_WFMT_AFFINE8 || wfmt == DSM_WFMT_AFFINE4) {
    if (cudaMemsetAsync(header, 0, sizeof(float) * n_experts, s) != cudaSuccess) return check_launch("memset");
    const int64_t gpe = int64_t(rows) * (cols / group_size);
    dim3 grid(unsigned(std::min<int64_t>(ceil_div(gpe, 256), 1024)), unsigned(n_experts));
    affine_amax_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(scales),
                                           static_cast<const __nv_bfloat16*>(biases), gpe,
                                           wfmt == DSM_WFMT_AFFINE8 ? 255.f : 15.f, header);
    if (int rc = check_launch("affine_amax")) return rc;
  } else if (wfmt == DSM_WFMT_FP4_G32) {
    if (cudaMemcpyAsync(header, tensor_scale, sizeof(float) * n_experts, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return check_launch("copy tensor scale");
  } else {
    fill_header_kernel<<<unsigned(ceil_div(n_experts, 256)), 256, 0, s>>>(header, n_experts, 1.f);
    if (int rc = check_launch("fill_header")) return rc;
  }
  PackArgs a;
  a.wfmt = wfmt;
  a.n_experts = n_experts;
  a.rows = rows;
  a.cols = cols;
  a.group_size = group_size > 0 ? group_size : 64;
  a.rt_count = int(ceil_div(rows, kTileRows));
  a.kc_count = int(ceil_div(cols, kChunkK));
  a.codes = codes;
  a.scales = scales;
  a.biases = biases;
  a.header = header;
  a.tiles = static_cast<uint8_t*>(packed) + packed_header_bytes(n_experts);
  a.src_dtype = src_dtype;
  const int64_t tiles = int64_t(n_experts) * a.rt_count * a.kc_count;
  pack_tiles_kernel<<<unsigned(tiles), 256, 0, s>>>(a);
  if (int rc = check_launch("pack_tiles")) return rc;
  if (wfmt == DSM_WFMT_F16 || wfmt == DSM_WFMT_AFFINE8 || wfmt == DSM_WFMT_AFFINE4) {
    finalize_prescale_header_kernel<<<unsigned(ceil_div(n_experts, 256)), 256, 0, s>>>(header, n_experts);
    return check_launch("finalize_header");
  }
  return DSM_OK;
}

extern "C" int dsm_affine_quantize(const void* w, int w_dtype, int64_t n_rows, int cols, int group_size, int bits,
                                   uint8_t* codes, void* scales, void* biases, void* stream) {
  using namespace dsm;
  DSM_REQUIRE(bits == 4 || bits == 8, "dsm_affine_quantize: bits must be 4 or 8");
  DSM_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, "dsm_affine_quantize: group_size 32/64/128");
  DSM_REQUIRE(cols > 0 && cols % group_size == 0, "dsm_affine_quantize: cols must be a multiple of group_size");
  DSM_REQUIRE(w_dtype == DSM_DT_F32 || w_dtype == DSM_DT_BF16, "dsm_affine_quantize: w must be F32 or BF16");
  DSM_REQUIRE(n_rows >= 0, "dsm_affine_quantize: bad shape");
  if (n_rows == 0) return DSM_OK;
  DSM_REQUIRE(w && codes && scales && biases, "dsm_affine_quantize: NULL pointer");
  const int64_t n_groups = n_rows * (cols / group_size);
  const unsigned blocks = unsigned(ceil_div(n_groups, 256));
  cudaStream_t s = as_stream(stream);
  if (w_dtype == DSM_DT_BF16)
    affine_quantize_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(w), n_rows, cols, group_size, bits, codes,
        static_cast<__nv_bfloat16*>(scales), static_cast<__nv_bfloat16*>(biases));
  else
    affine_quantize_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(w), n_rows, cols, group_size, bits,
                                                          codes, static_cast<float*>(scales), static_cast<float*>(biases));
  return check_launch("affine_quantize");
}
