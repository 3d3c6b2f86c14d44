// INT4 group-32 quantization, 144-byte super-block packing and bit-exact
// dequantization kernels (sm_100a), plus the library's host helpers.
//
// Reference semantics: antigravity-engine/src/dequant.py (quantize_weights_int4
// :22-60, repack_to_superblocks :69-132, unpack_superblock :135-156,
// lut_dequantize / arithmetic_dequantize :183-252), src/dequant.py
// (quantize_fp16_to_int4 :26-55, lut_dequantize_fp16 :79-113,
// unpack_superblock_weights :116-147). All of them are byte / HBM streaming work:
// coalesced 16-byte loads and stores, grids sized in whole waves of the SM count.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace mb {

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
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

bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_tmap_3d_u8(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides[2],
                       const uint32_t box[3]) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides[0], strides[1]};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), d, st, b, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static inline int grid_for(int64_t work, int per_block) {
  int64_t b = (work + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 32;
  if (b > cap) b = cap;
  return static_cast<int>(b < 1 ? 1 : b);
}

// ---------------------------------------------------------------------------
// Quantize: one warp per group of 32 consecutive weights.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float nanmax(float a, float b) {  // NaN-propagating like np.max
  return (b > a || b != b) ? b : a;
}

__global__ void __launch_bounds__(256) k_quantize(const void* __restrict__ w, int w_is_fp16, int64_t ngroups,
                                                  int variant, int8_t* __restrict__ q_out,
                                                  uint16_t* __restrict__ s_out, uint8_t* __restrict__ sb_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < ngroups;
       g += warps) {
    const int64_t i = g * 32 + lane;
    float x = w_is_fp16 ? __half2float(__ushort_as_half(static_cast<const uint16_t*>(w)[i]))
                        : static_cast<const float*>(w)[i];
    float a = fabsf(x);
#pragma unroll
    for (int o = 16; o; o >>= 1) a = nanmax(a, __shfl_xor_sync(0xffffffffu, a, o));
    // scale = alpha / 7 in fp32 (1.0 for a zero group), stored as fp16
    const float s32 = (a == 0.0f) ? 1.0f : __fdiv_rn(a, 7.0f);
    const __half s16 = __float2half_rn(s32);
    const float div = (variant == 0) ? __half2float(s16) : s32;
    float r = rintf(__fdiv_rn(x, div));  // round half to even, IEEE divide
    int qi;
    if (r != r) {
      qi = 0;  // NaN casts to 0 on the reference's host (x86 cvt + int8 truncation)
    } else {
      r = fminf(fmaxf(r, -8.0f), 7.0f);
      qi = static_cast<int>(r);
    }
    if (q_out) q_out[i] = static_cast<int8_t>(qi);
    if (s_out && lane == 0) s_out[g] = __half_as_ushort(s16);
    if (sb_out) {
      const int64_t sb = g >> 3;
      const int gi = static_cast<int>(g & 7);
      uint8_t* base = sb_out + sb * 144;
      const int nib = (qi + 8) & 0xF;
      const int hi = __shfl_down_sync(0xffffffffu, nib, 1);
      if ((lane & 1) == 0) base[16 + gi * 16 + (lane >> 1)] = static_cast<uint8_t>(nib | (hi << 4));
      if (lane == 0) {
        const uint16_t sb16 = __half_as_ushort(s16);
        base[2 * gi] = static_cast<uint8_t>(sb16 & 0xFF);
        base[2 * gi + 1] = static_cast<uint8_t>(sb16 >> 8);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Pack int8 q + fp16 scales -> super-blocks. One thread per 16-byte chunk of the
// output (9 chunks per super-block: chunk 0 = scales, chunk c = group c-1's nibbles).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_pack(const int8_t* __restrict__ q, const uint16_t* __restrict__ s,
                                              int64_t nsb, uint8_t* __restrict__ out) {
  const int64_t total = nsb * 9;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t sb = t / 9;
    const int c = static_cast<int>(t % 9);
    uint4 v;
    if (c == 0) {
      v = *reinterpret_cast<const uint4*>(s + sb * 8);  // 8 scales, 16 bytes
    } else {
      const int4 raw0 = *reinterpret_cast<const int4*>(q + sb * 256 + (c - 1) * 32);
      const int4 raw1 = *reinterpret_cast<const int4*>(q + sb * 256 + (c - 1) * 32 + 16);
      const uint32_t in[8] = {(uint32_t)raw0.x, (uint32_t)raw0.y, (uint32_t)raw0.z, (uint32_t)raw0.w,
                              (uint32_t)raw1.x, (uint32_t)raw1.y, (uint32_t)raw1.z, (uint32_t)raw1.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // 8 int8 values (two input words) -> 4 bytes of nibble pairs, each nibble q+8
        const uint32_t a = in[2 * j] ^ 0x08080808u, b = in[2 * j + 1] ^ 0x08080808u;
        // (q + 8) & 0xF == (q ^ 8) & 0xF for q in [-8, 7]
        const uint32_t a0 = a & 0x0F0F0F0Fu, b0 = b & 0x0F0F0F0Fu;
        // byte pairs (e0,e1),(e2,e3): low | high << 4
        const uint32_t pa = (a0 & 0x000F000Fu) | ((a0 >> 4) & 0x00F000F0u);
        const uint32_t pb = (b0 & 0x000F000Fu) | ((b0 >> 4) & 0x00F000F0u);
        // pa bytes: [e0|e1<<4, -, e2|e3<<4, -] -> gather bytes 0 and 2
        o[j] = prmt(pa, pb, 0x6420u);
      }
      v = make_uint4(o[0], o[1], o[2], o[3]);
    }
    *reinterpret_cast<uint4*>(out + sb * 144 + c * 16) = v;
  }
}

// ---------------------------------------------------------------------------
// Unpack super-blocks -> int8 q and fp16 scales.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_unpack(const uint8_t* __restrict__ sbp, int64_t nsb, int8_t* __restrict__ q,
                                                uint16_t* __restrict__ s) {
  const int64_t total = nsb * 9;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t sb = t / 9;
    const int c = static_cast<int>(t % 9);
    const uint4 v = *reinterpret_cast<const uint4*>(sbp + sb * 144 + c * 16);
    if (c == 0) {
      if (s) *reinterpret_cast<uint4*>(s + sb * 8) = v;
    } else if (q) {
      const uint32_t in[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t lo = in[j] & 0x0F0F0F0Fu, hi = (in[j] >> 4) & 0x0F0F0F0Fu;
        // interleave low/high nibbles of each byte: e(2i) = lo byte i, e(2i+1) = hi byte i
        o[2 * j] = __vsub4(prmt(lo, hi, 0x5140u), 0x08080808u);      // bytes: lo0 hi0 lo1 hi1
        o[2 * j + 1] = __vsub4(prmt(lo, hi, 0x7362u), 0x08080808u);  // bytes: lo2 hi2 lo3 hi3 (per-byte, no borrow)
      }
      int8_t* dst = q + sb * 256 + (c - 1) * 32;
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(dst + 16) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  }
}

// ---------------------------------------------------------------------------
// Dequant super-blocks -> fp16. One thread per (super-block, group): a 16-byte
// nibble load + its scale -> 32 fp16 = four 16-byte stores.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_h2(uint16_t lo, uint16_t hi) { return lo | (static_cast<uint32_t>(hi) << 16); }

// 4 nibble bytes (8 elements, element 2j in the low nibble of byte j) -> 4 half2
// in element order, each scaled by s2 with one rounding.
__device__ __forceinline__ void expand_word(uint32_t wd, uint32_t s2, uint32_t* o) {
  // element order: (e0,e1) (e2,e3) (e4,e5) (e6,e7); nibbles_to_half2 pairs bytes 0/2.
  uint32_t lo02, hi02, lo13, hi13;
  nibbles_to_half2(wd, lo02, hi02);       // lo02 = (e0, e4), hi02 = (e1, e5)
  nibbles_to_half2(wd >> 8, lo13, hi13);  // lo13 = (e2, e6), hi13 = (e3, e7)
  o[0] = hmul2(prmt(lo02, hi02, 0x5410u), s2);  // (e0, e1)
  o[1] = hmul2(prmt(lo13, hi13, 0x5410u), s2);  // (e2, e3)
  o[2] = hmul2(prmt(lo02, hi02, 0x7632u), s2);  // (e4, e5)
  o[3] = hmul2(prmt(lo13, hi13, 0x7632u), s2);  // (e6, e7)
}

__global__ void __launch_bounds__(256) k_dequant(const uint8_t* __restrict__ sbp, int64_t nsb,
                                                 uint16_t* __restrict__ out) {
  const int64_t total = nsb * 8;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t sb = t >> 3;
    const int g = static_cast<int>(t & 7);
    const uint8_t* base = sbp + sb * 144;
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(base + 16 + g * 16));
    const uint16_t s = __ldg(reinterpret_cast<const unsigned short*>(base) + g);
    const uint32_t s2 = pack_h2(s, s);
    uint32_t o[16];
    expand_word(v.x, s2, o);
    expand_word(v.y, s2, o + 4);
    expand_word(v.z, s2, o + 8);
    expand_word(v.w, s2, o + 12);
    uint4* dst = reinterpret_cast<uint4*>(out + sb * 256 + g * 32);
    __stcs(dst + 0, make_uint4(o[0], o[1], o[2], o[3]));
    __stcs(dst + 1, make_uint4(o[4], o[5], o[6], o[7]));
    __stcs(dst + 2, make_uint4(o[8], o[9], o[10], o[11]));
    __stcs(dst + 3, make_uint4(o[12], o[13], o[14], o[15]));
  }
}

// int8 q + fp16 scales (arbitrary group size) -> fp16, fp16(q * s) with one rounding.
__global__ void __launch_bounds__(256) k_dequant_q(const int8_t* __restrict__ q, const uint16_t* __restrict__ s,
                                                   int64_t n, int group, uint16_t* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const __half sc = __ushort_as_half(s[i / group]);
    out[i] = __half_as_ushort(__hmul(__int2half_rn(static_cast<int>(q[i])), sc));
  }
}

__global__ void __launch_bounds__(256) k_lut_gather(const int32_t* __restrict__ idx, int64_t n,
                                                    const uint16_t* __restrict__ lut, int64_t rows, int cols,
                                                    int64_t group_len, uint16_t* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int j = idx[i];
    j = j < 0 ? 0 : (j >= cols ? cols - 1 : j);
    const int64_t r = (i / group_len) % rows;
    out[i] = lut[r * cols + j];
  }
}

// Column extract: one thread per 32-wide group of the output [K, c1-c0] weight.
__global__ void __launch_bounds__(256) k_extract_cols(const uint8_t* __restrict__ sbp, int K, int M, int c0, int Ms,
                                                      uint8_t* __restrict__ out) {
  const int gpr = Ms / 32;  // groups per output row
  const int64_t total = static_cast<int64_t>(K) * gpr;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t k = t / gpr;
    const int gcol = static_cast<int>(t % gpr);
    const int64_t src_flat = k * M + c0 + gcol * 32;  // group-aligned
    const int64_t dst_flat = k * Ms + gcol * 32;
    const uint8_t* sb = sbp + (src_flat >> 8) * 144;
    const int sg = static_cast<int>((src_flat & 255) >> 5);
    uint8_t* db = out + (dst_flat >> 8) * 144;
    const int dg = static_cast<int>((dst_flat & 255) >> 5);
    *reinterpret_cast<uint4*>(db + 16 + dg * 16) = *reinterpret_cast<const uint4*>(sb + 16 + sg * 16);
    *reinterpret_cast<uint16_t*>(db + 2 * dg) = *reinterpret_cast<const uint16_t*>(sb + 2 * sg);
  }
}

}  // namespace mb

using namespace mb;

extern "C" {

int32_t mb_abi_version(void) { return MB_ABI_VERSION; }

const char* mb_status_string(int32_t s) {
  switch (s) {
    case MB_OK: return "ok";
    case MB_ERR_NULL: return "null pointer";
    case MB_ERR_ARGS: return "invalid arguments";
    case MB_ERR_WORKSPACE: return "workspace too small";
    case MB_ERR_LAUNCH: return "CUDA launch failed";
    case MB_ERR_ALIGN: return "pointer not 16-byte aligned";
    case MB_ERR_UNSUPPORTED: return "unsupported shape";
    default: return "unknown status";
  }
}

int32_t mb_int4_quantize(const void* w, int32_t w_is_fp16, int64_t n, int32_t variant, int8_t* q_out,
                         uint16_t* scales_out, uint8_t* sb_out, void* stream) {
  if (n < 0 || n % 32 != 0 || (sb_out && n % 256 != 0) || (variant != 0 && variant != 1)) return MB_ERR_ARGS;
  if (n == 0) return MB_OK;
  if (!w || (!q_out && !scales_out && !sb_out)) return MB_ERR_NULL;
  const int64_t ngroups = n / 32;
  k_quantize<<<grid_for(ngroups, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(w, w_is_fp16, ngroups, variant,
                                                                                  q_out, scales_out, sb_out);
  return launch_status();
}

int32_t mb_int4_pack(const int8_t* q, const uint16_t* scales, int64_t n, uint8_t* sb_out, void* stream) {
  if (n < 0 || n % 256 != 0) return MB_ERR_ARGS;
  if (n == 0) return MB_OK;
  if (!q || !scales || !sb_out) return MB_ERR_NULL;
  if (!aligned(q, 16) || !aligned(scales, 16) || !aligned(sb_out, 16)) return MB_ERR_ALIGN;
  const int64_t nsb = n / 256;
  k_pack<<<grid_for(nsb * 9, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(q, scales, nsb, sb_out);
  return launch_status();
}

int32_t mb_int4_unpack(const uint8_t* sb, int64_t nsb, int8_t* q_out, uint16_t* scales_out, void* stream) {
  if (nsb < 0) return MB_ERR_ARGS;
  if (nsb == 0) return MB_OK;
  if (!sb || (!q_out && !scales_out)) return MB_ERR_NULL;
  if (!aligned(sb, 16) || (q_out && !aligned(q_out, 16)) || (scales_out && !aligned(scales_out, 16)))
    return MB_ERR_ALIGN;
  k_unpack<<<grid_for(nsb * 9, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(sb, nsb, q_out, scales_out);
  return launch_status();
}

int32_t mb_int4_dequant(const uint8_t* sb, uint16_t* out, int64_t nsb, void* stream) {
  if (nsb < 0) return MB_ERR_ARGS;
  if (nsb == 0) return MB_OK;
  if (!sb || !out) return MB_ERR_NULL;
  if (!aligned(sb, 16) || !aligned(out, 16)) return MB_ERR_ALIGN;
  k_dequant<<<grid_for(nsb * 8, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(sb, nsb, out);
  return launch_status();
}

int32_t mb_int4_dequant_q(const int8_t* q, const uint16_t* scales, int64_t n, int32_t group, uint16_t* out,
                          void* stream) {
  if (n < 0 || group < 1 || n % group != 0) return MB_ERR_ARGS;
  if (n == 0) return MB_OK;
  if (!q || !scales || !out) return MB_ERR_NULL;
  k_dequant_q<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(q, scales, n, group, out);
  return launch_status();
}

int32_t mb_lut_gather_f16(const int32_t* idx, int64_t n, const uint16_t* lut, int64_t lut_rows, int32_t lut_cols,
                          int64_t group_len, uint16_t* out, void* stream) {
  if (n < 0 || lut_rows < 1 || lut_cols < 1 || group_len < 1) return MB_ERR_ARGS;
  if (n == 0) return MB_OK;
  if (!idx || !lut || !out) return MB_ERR_NULL;
  k_lut_gather<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(idx, n, lut, lut_rows, lut_cols,
                                                                                group_len, out);
  return launch_status();
}

int32_t mb_int4_extract_columns(const uint8_t* sb, int32_t K, int32_t M, int32_t c0, int32_t c1, uint8_t* out,
                                void* stream) {
  if (!sb || !out) return MB_ERR_NULL;
  if (K < 1 || M < 32 || M % 32 != 0 || c0 < 0 || c1 > M || c1 <= c0 || c0 % 32 != 0 || c1 % 32 != 0)
    return MB_ERR_ARGS;
  const int64_t Ms = c1 - c0;
  if ((static_cast<int64_t>(K) * Ms) % 256 != 0 || (static_cast<int64_t>(K) * M) % 256 != 0) return MB_ERR_ARGS;
  if (!aligned(sb, 16) || !aligned(out, 16)) return MB_ERR_ALIGN;
  const int64_t total = static_cast<int64_t>(K) * (Ms / 32);
  k_extract_cols<<<grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(sb, K, M, c0,
                                                                                      static_cast<int>(Ms), out);
  return launch_status();
}

}  // extern "C"
