// Fused INT4 super-block batched GEMM for B200 (sm_100a):
//   out[N, M] (fp16) = act[N, K] (fp16) x dequant(sb)[K, M], fp32 accumulation.
//
// Replaces the reference's batched_gemm entry point (Metal batched_gemm_simdgroup /
// fused_batched_gemm_int4, antigravity-engine/src/shaders/batched_gemm.metal:74-169;
// CPU form `activations @ W`, batch_generator.py:290). The weight stream is the
// reference's 144-byte super-block format, read in place.
//
// Design (weight streaming, HBM bound):
//  * The M columns are cut into strips of WS = 256 (one super-block per row) or 128
//    columns. Each strip is handled by one thread-block cluster of Ck CTAs that
//    split its K rows; the grid (strips x Ck) is sized to one wave of the SMs. The
//    split-K partial sums are reduced on chip through distributed shared memory at
//    the end, so there is no global workspace, no atomics, and the result is
//    deterministic.
//  * One producer thread per CTA streams the strip's super-block rows with 3-D TMA
//    tile loads (cp.async.bulk.tensor, L2 evict-first) into a ring of shared-memory
//    stages guarded by mbarriers. The weights never depend on the previous kernel,
//    so the whole ring is filled before griddepcontrol.wait (programmatic dependent
//    launch): a CTA of the next call, resident beside this one, prefetches while this
//    one computes.
//  * After griddepcontrol.wait the consumer warps stage the CTA's activation slice in
//    shared memory (one pass, L2 resident) and expand nibbles straight into
//    mma.m16n8k16 A fragments in registers: byte permute + magic-exponent fp16
//    conversion + one fp16 multiply by the group scale, bit-exact with the reference
//    dequant; the batch (padded to 8/16/32) is the MMA n dimension, fp32 accumulate.
//  * Shared-memory rows are laid out so the fragment loads are bank-conflict free:
//    full 144-byte super-block rows (WS = 256), or a 16-byte scale row plus a
//    nibble row padded to 80 / 96 bytes by the TMA box (WS = 128, M % 256 == 128).
#include <algorithm>

#include "common.cuh"
#include "gemm_tc.cuh"

namespace mb {

constexpr int kSB = 144;        // bytes per super-block
constexpr int kSliceRows = 16;  // k rows per MMA slice
constexpr int kSPS = 8;         // slices per full stage (128 rows)
constexpr int kStageRows = kSPS * kSliceRows;
constexpr int kMaxStages = 8;
constexpr int kMaxCk = 8;

// Shared-memory layout of one pipeline stage (128 rows of the CTA's strip).
//  WS = 256: full 144-byte super-block rows (scales then nibbles), row stride 144 B.
//  WS = 128 / 64: a 16-byte scale row per k row, then the strip's nibble bytes in a
//  row padded by the TMA box (80 / 48 bytes for one row phase, 96 / 32 bytes for two)
//  so that the fragment loads below hit 32 distinct banks. With P = 2 row phases
//  (M % 256 == 128) rows of each phase are stored together.
template <int WS, int P>
struct Layout {
  static_assert(WS == 256 || WS == 128, "strip width");
  static_assert(WS != 256 || P == 1, "a 256-wide strip needs M % 256 == 0");
  static_assert(P == 1 || P == 2, "row phases");
  static constexpr int kNibRow = (WS == 128) ? (P == 1 ? 80 : 96) : (P == 1 ? 48 : 32);
  static constexpr int kScRegion = kStageRows * 16;
  static constexpr int kStageBytes = (WS == 256) ? kStageRows * kSB : kStageRows * (16 + kNibRow);
  static constexpr int kRowsPerPhase = kStageRows / P;
  static __device__ __host__ constexpr int bytes(int n) {  // tx bytes of a stage with n slices
    return (WS == 256) ? n * kSliceRows * kSB : n * kSliceRows * (16 + kNibRow);
  }
  // byte offset of row k's scale chunk / first strip nibble byte within a stage
  static __device__ __forceinline__ constexpr int sc(int k) {
    return (WS == 256) ? k * kSB : ((k & (P - 1)) * kRowsPerPhase + k / P) * 16;
  }
  static __device__ __forceinline__ constexpr int nib(int k) {
    return (WS == 256) ? k * kSB + 16 : kScRegion + ((k & (P - 1)) * kRowsPerPhase + k / P) * kNibRow;
  }
};

struct GemmParams {
  uint16_t* out;        // [N, M] fp16
  const uint16_t* act;  // [N, K] fp16
  uint32_t* err;        // optional device error word (may be null)
  int N, K, M;
  int KS;               // k slices (ceil(K / 16))
  int Ck;               // CTAs per cluster = K split
  int S;                // stages in the ring
  int xstride;          // bytes per activation row in shared memory
  int xbytes;           // activation region
};

struct WMaps {  // weight tensor maps: full-stage and 16-row boxes (scale / nibble rows)
  CUtensorMap full_a, full_b, slice_a, slice_b;
};

template <int NW>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t (&w)[NW]) {
  if constexpr (NW == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (NW == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}
__device__ __forceinline__ uint32_t lds_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// One 16-row k slice for this thread's MR-column run.
// Thread (g4 = lane/4, t4 = lane%4) owns rows 2t4, 2t4+1, 2t4+8, 2t4+9 of the slice
// (the k positions of the m16n8k16 A fragment) and MR consecutive columns; m16 tile
// i of the warp maps fragment row g4 to column 2i and row g4+8 to column 2i+1 of the
// run, so each nibble byte feeds exactly one tile and the warp has MR/2 independent
// accumulator chains per batch tile. The weight operand is fp16((n - 8) * s): exact
// magic-exponent conversion of the nibble, then one rounding multiply by the group
// scale — bit-identical to the reference dequant.
//   stage, k0: stage base and the stage-local row 2t4 of this slice; nb: byte offset
//   of the run within a nibble row; ge / go: scale index for even / odd rows;
//   xrow: this lane's activation row (n = 8 nt + g4) at the slice's first k.
template <int NT, int WS, int P, int MR>
__device__ __forceinline__ void consume_slice(const uint8_t* stage, int k0, int nb, int ge, int go,
                                              const uint8_t* const (&xrow)[NT], const bool (&xok)[NT], int t4,
                                              float (&acc)[MR / 2][NT][4]) {
  using L = Layout<WS, P>;
  constexpr int NW = MR / 8;  // 32-bit nibble words per row
  // rows 2t4, 2t4+1, 2t4+8, 2t4+9 as constant offsets from row 2t4
  constexpr int dn1 = L::nib(1) - L::nib(0), dn8 = L::nib(8) - L::nib(0), dn9 = L::nib(9) - L::nib(0);
  constexpr int ds1 = L::sc(1) - L::sc(0), ds8 = L::sc(8) - L::sc(0), ds9 = L::sc(9) - L::sc(0);
  const uint8_t* pn = stage + L::nib(k0) + nb;
  const uint8_t* ps = stage + L::sc(k0);
  uint32_t w0[NW], w1[NW], w2[NW], w3[NW];
  lds_words<NW>(pn, w0);
  lds_words<NW>(pn + dn1, w1);
  lds_words<NW>(pn + dn8, w2);
  lds_words<NW>(pn + dn9, w3);
  const uint32_t s01 = lds_u16(ps + 2 * ge) | (lds_u16(ps + ds1 + 2 * go) << 16);
  const uint32_t s23 = lds_u16(ps + ds8 + 2 * ge) | (lds_u16(ps + ds9 + 2 * go) << 16);
  uint32_t bf[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    bf[nt][0] = xok[nt] ? lds_u32(xrow[nt] + 4 * t4) : 0u;
    bf[nt][1] = xok[nt] ? lds_u32(xrow[nt] + 16 + 4 * t4) : 0u;
  }
#pragma unroll
  for (int v = 0; v < NW; ++v) {
    const uint32_t p01l = prmt(w0[v], w1[v], 0x5410u), p01h = prmt(w0[v], w1[v], 0x7632u);
    const uint32_t p23l = prmt(w2[v], w3[v], 0x5410u), p23h = prmt(w2[v], w3[v], 0x7632u);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t q01 = ((b & 2) ? p01h : p01l) >> (8 * (b & 1));
      const uint32_t q23 = ((b & 2) ? p23h : p23l) >> (8 * (b & 1));
      uint32_t a0, a1, a2, a3;
      nibbles_to_half2(q01, a0, a1);
      nibbles_to_half2(q23, a2, a3);
      a0 = hmul2(a0, s01);
      a1 = hmul2(a1, s01);
      a2 = hmul2(a2, s23);
      a3 = hmul2(a3, s23);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_16816(acc[4 * v + b][nt], a0, a1, a2, a3, bf[nt][0], bf[nt][1]);
    }
  }
}

// The same slice computation split in two halves, so a caller can load slice i + 1
// (after waiting for its stage) before it computes slice i from registers: the
// shared-memory latency of one slice overlaps the arithmetic of the previous one.
template <int NT, int MR>
struct SliceRegs {
  uint32_t w0[MR / 8], w1[MR / 8], w2[MR / 8], w3[MR / 8];
  uint32_t s01, s23;
  uint32_t bf[NT][2];
};

template <int NT, int WS, int P, int MR>
__device__ __forceinline__ void load_slice(const uint8_t* stage, int k0, int nb, int ge, int go,
                                           const uint8_t* const (&xrow)[NT], const bool (&xok)[NT], int t4,
                                           SliceRegs<NT, MR>& r) {
  using L = Layout<WS, P>;
  constexpr int NW = MR / 8;
  constexpr int dn1 = L::nib(1) - L::nib(0), dn8 = L::nib(8) - L::nib(0), dn9 = L::nib(9) - L::nib(0);
  constexpr int ds1 = L::sc(1) - L::sc(0), ds8 = L::sc(8) - L::sc(0), ds9 = L::sc(9) - L::sc(0);
  const uint8_t* pn = stage + L::nib(k0) + nb;
  const uint8_t* ps = stage + L::sc(k0);
  lds_words<NW>(pn, r.w0);
  lds_words<NW>(pn + dn1, r.w1);
  lds_words<NW>(pn + dn8, r.w2);
  lds_words<NW>(pn + dn9, r.w3);
  r.s01 = lds_u16(ps + 2 * ge) | (lds_u16(ps + ds1 + 2 * go) << 16);
  r.s23 = lds_u16(ps + ds8 + 2 * ge) | (lds_u16(ps + ds9 + 2 * go) << 16);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    r.bf[nt][0] = xok[nt] ? lds_u32(xrow[nt] + 4 * t4) : 0u;
    r.bf[nt][1] = xok[nt] ? lds_u32(xrow[nt] + 16 + 4 * t4) : 0u;
  }
}

template <int NT, int MR>
__device__ __forceinline__ void compute_slice(const SliceRegs<NT, MR>& r, float (&acc)[MR / 2][NT][4]) {
  constexpr int NW = MR / 8;
#pragma unroll
  for (int v = 0; v < NW; ++v) {
    const uint32_t p01l = prmt(r.w0[v], r.w1[v], 0x5410u), p01h = prmt(r.w0[v], r.w1[v], 0x7632u);
    const uint32_t p23l = prmt(r.w2[v], r.w3[v], 0x5410u), p23h = prmt(r.w2[v], r.w3[v], 0x7632u);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t q01 = ((b & 2) ? p01h : p01l) >> (8 * (b & 1));
      const uint32_t q23 = ((b & 2) ? p23h : p23l) >> (8 * (b & 1));
      uint32_t a0, a1, a2, a3;
      nibbles_to_half2(q01, a0, a1);
      nibbles_to_half2(q23, a2, a3);
      a0 = hmul2(a0, r.s01);
      a1 = hmul2(a1, r.s01);
      a2 = hmul2(a2, r.s23);
      a3 = hmul2(a3, r.s23);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_16816(acc[4 * v + b][nt], a0, a1, a2, a3, r.bf[nt][0], r.bf[nt][1]);
    }
  }
}

// Scale folded into the conversion: the A operand is fp16(n * s) for the raw nibble
// n in [0, 15] -- one lop3 and one fma.rn.f16x2 per two weights, with n * s rounded
// once -- and the -8 offset is applied after the MMAs through a correction tile:
// corr[m][n] = sum_k s[k][group(m)] x[n][k] (one MMA per slice whose A fragment is the
// scale pairs already in registers), out = acc - 8 corr. All columns of one thread
// run share a group, so one correction tile serves every tile of the run.
template <int NT, int MR>
__device__ __forceinline__ void compute_slice_folded(const SliceRegs<NT, MR>& r, float (&acc)[MR / 2][NT][4],
                                                     float (&corr)[NT][4]) {
  constexpr int NW = MR / 8;
  // per-half constants: (1024 + n) * s - 1024 s and (1024 + 16 n) * s / 16 - 64 s
  const uint32_t s01n = r.s01 ^ 0x80008000u, s23n = r.s23 ^ 0x80008000u;  // -s
  uint32_t c01lo, c23lo, c01hi, c23hi, s01q, s23q;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(c01lo) : "r"(s01n), "r"(0x64006400u));  // -1024 s (exact)
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(c23lo) : "r"(s23n), "r"(0x64006400u));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(c01hi) : "r"(s01n), "r"(0x54005400u));  // -64 s (exact)
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(c23hi) : "r"(s23n), "r"(0x54005400u));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(s01q) : "r"(r.s01), "r"(0x2C002C00u));   // s / 16 (exact)
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(s23q) : "r"(r.s23), "r"(0x2C002C00u));
#pragma unroll
  for (int v = 0; v < NW; ++v) {
    const uint32_t p01l = prmt(r.w0[v], r.w1[v], 0x5410u), p01h = prmt(r.w0[v], r.w1[v], 0x7632u);
    const uint32_t p23l = prmt(r.w2[v], r.w3[v], 0x5410u), p23h = prmt(r.w2[v], r.w3[v], 0x7632u);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t q01 = ((b & 2) ? p01h : p01l) >> (8 * (b & 1));
      const uint32_t q23 = ((b & 2) ? p23h : p23l) >> (8 * (b & 1));
      uint32_t a0, a1, a2, a3;
      const uint32_t l01 = lop3<0xEA>(q01, 0x000F000Fu, 0x64006400u), h01 = lop3<0xEA>(q01, 0x00F000F0u, 0x64006400u);
      const uint32_t l23 = lop3<0xEA>(q23, 0x000F000Fu, 0x64006400u), h23 = lop3<0xEA>(q23, 0x00F000F0u, 0x64006400u);
      asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(a0) : "r"(l01), "r"(r.s01), "r"(c01lo));
      asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(a1) : "r"(h01), "r"(s01q), "r"(c01hi));
      asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(a2) : "r"(l23), "r"(r.s23), "r"(c23lo));
      asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(a3) : "r"(h23), "r"(s23q), "r"(c23hi));
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_16816(acc[4 * v + b][nt], a0, a1, a2, a3, r.bf[nt][0], r.bf[nt][1]);
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) mma_16816(corr[nt], r.s01, r.s01, r.s23, r.s23, r.bf[nt][0], r.bf[nt][1]);
}

template <int WS, int P>
__device__ __forceinline__ void issue_stage(const WMaps& maps, uint8_t* dst, uint64_t* bar, int k0, int n,
                                            const int (&ey)[P], const int (&ex)[P], uint64_t pol) {
  using L = Layout<WS, P>;
  mbar_expect_tx(bar, L::bytes(n));
  if constexpr (WS == 256) {
    if (n == kSPS) {
      tma_load_3d(dst, &maps.full_a, bar, 0, ey[0], k0, pol);
    } else {
      for (int j = 0; j < n; ++j)
        tma_load_3d(dst + j * kSliceRows * kSB, &maps.slice_a, bar, 0, ey[0], k0 + j * kSliceRows, pol);
    }
  } else {
    constexpr int rp = L::kRowsPerPhase;
#pragma unroll
    for (int r = 0; r < P; ++r) {
      uint8_t* sdst = dst + r * rp * 16;
      uint8_t* ndst = dst + L::kScRegion + r * rp * L::kNibRow;
      if (n == kSPS) {
        tma_load_3d(sdst, &maps.full_a, bar, 0, ey[r], k0 / P, pol);
        tma_load_3d(ndst, &maps.full_b, bar, ex[r], ey[r], k0 / P, pol);
      } else {
        constexpr int sp = kSliceRows / P;
        for (int j = 0; j < n; ++j) {
          tma_load_3d(sdst + j * sp * 16, &maps.slice_a, bar, 0, ey[r], (k0 + j * kSliceRows) / P, pol);
          tma_load_3d(ndst + j * sp * L::kNibRow, &maps.slice_b, bar, ex[r], ey[r], (k0 + j * kSliceRows) / P, pol);
        }
      }
    }
  }
}

__device__ __forceinline__ void store_half2(uint16_t* dst, float a, float b) {
  const __half2 x = __floats2half2_rn(a, b);
  *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(&x);
}

// Columns per thread run for (NT, WS): 32 / NT, at most WS / 8 (eight runs per warp).
template <int NT, int WS>
struct RunCols {
  static constexpr int v = (32 / NT < WS / 8) ? 32 / NT : WS / 8;
};

// NT: n-tiles of 8 batch rows (1, 2, 4); WS: strip width; P: row phases (1, 2);
// CW: consumer warps. __launch_bounds__(.., 2): a CTA uses at most half an SM's
// registers so the next call's CTAs (launched early through PDL) can be resident
// and prefetch their weights while this one computes.
template <int NT, int WS, int P, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 2)
    k_gemm_int4(const __grid_constant__ WMaps maps, const GemmParams p) {
  using L = Layout<WS, P>;
  constexpr int MR = RunCols<NT, WS>::v;  // columns per thread run
  constexpr int kTiles = MR / 2;          // m16 tiles per warp
  constexpr int kCm = WS / (8 * MR);      // column parts per strip (one warp each)
  constexpr int kKG = CW / kCm;           // warps sharing a column part (k groups)
  static_assert(kCm * kKG == CW, "warp layout");
  constexpr int kRegs = kTiles * NT * 4;  // accumulators per thread
  constexpr int kThreads = (CW + 1) * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* xs = stages + p.S * L::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(xs + p.xbytes);
  uint64_t* empty = full + kMaxStages;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int strip = blockIdx.x / p.Ck;
  const int q = blockIdx.x - strip * p.Ck;  // == rank in the cluster (cluster dims = (Ck,1,1))
  const int sl0 = static_cast<int>((static_cast<long long>(q) * p.KS) / p.Ck);
  const int sl1 = static_cast<int>((static_cast<long long>(q + 1) * p.KS) / p.Ck);
  const int nst = (sl1 - sl0 + kSPS - 1) / kSPS;
  const int c0 = strip * WS;
  // per row phase: super-block index within a period (y), first nibble byte of the
  // strip in that super-block (x) and the scale index of the strip's first column
  int ey[P], ex[P], grp[P];
#pragma unroll
  for (int r = 0; r < P; ++r) {
    const long long f = static_cast<long long>(r) * p.M + c0;
    ey[r] = static_cast<int>(f >> 8);
    const int e = static_cast<int>(f & 255);
    ex[r] = 16 + e / 2;
    grp[r] = e / 32;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, CW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  float* slots = reinterpret_cast<float*>(stages);  // final reduction scratch (ring + activations)
  if (warp == CW) {
    // ---------------- producer: weights only, no dependency on the previous grid ----
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      for (int st = 0; st < nst; ++st) {
        const int s = st % p.S;
        if (st >= p.S && !mbar_wait(empty + s, ((st / p.S) - 1) & 1) && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
        const int sl = sl0 + st * kSPS;
        issue_stage<WS, P>(maps, stages + s * L::kStageBytes, full + s, sl * kSliceRows, min(kSPS, sl1 - sl), ey, ex,
                           pol);
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    const int g4 = lane >> 2, t4 = lane & 3;
    const int mpart = warp % kCm, kg = warp / kCm;
    const int mcol = mpart * 8 * MR + g4 * MR;  // first column of this thread's run in the strip
    const int nb = (WS == 256) ? mcol / 2 : mcol / 2;
    const int ge = grp[0] + mcol / 32, go = grp[P - 1] + mcol / 32;

    pdl_wait();  // activations may come from the previous grid; all writes follow it
    // stage this CTA's activation slice [N][k0, k1) in shared memory (zero past K)
    const int k0 = sl0 * kSliceRows;
    const int chunks = (sl1 - sl0) * kSliceRows / 8;  // 16-byte chunks per row
    for (int idx = threadIdx.x; idx < p.N * chunks; idx += CW * 32) {
      const int n = idx / chunks, c = idx - n * chunks;
      const int k = k0 + c * 8;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (k < p.K) v = __ldg(reinterpret_cast<const uint4*>(p.act + static_cast<size_t>(n) * p.K + k));
      *reinterpret_cast<uint4*>(xs + n * p.xstride + c * 16) = v;
    }
    named_bar_sync(1, CW * 32);

    float acc[kTiles][NT][4];
#pragma unroll
    for (int i = 0; i < kTiles; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[i][nt][c] = 0.0f;
    bool xok[NT];
    const uint8_t* xbase[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nt * 8 + g4;
      xok[nt] = n < p.N;
      xbase[nt] = xs + (xok[nt] ? n : 0) * p.xstride;
    }

    for (int st = 0; st < nst; ++st) {
      const int s = st % p.S;
      if (!mbar_wait(full + s, (st / p.S) & 1) && lane == 0 && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
      const uint8_t* stage = stages + s * L::kStageBytes;
      const int n = min(kSPS, sl1 - (sl0 + st * kSPS));
      for (int j = kg; j < n; j += kKG) {
        const int kx = (st * kSPS + j) * kSliceRows;  // k offset within the activation slice
        const uint8_t* xr[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) xr[nt] = xbase[nt] + kx * 2;
        consume_slice<NT, WS, P, MR>(stage, j * kSliceRows + 2 * t4, nb, ge, go, xr, xok, t4, acc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);
    }

    // park the partial sums (lane-major: conflict free) once every warp is done with
    // the stage ring and the activation slice
    named_bar_sync(1, CW * 32);
    float* slot = slots + warp * kRegs * 32 + lane;
#pragma unroll
    for (int i = 0; i < kTiles; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) slot[((i * NT + nt) * 4 + c) * 32] = acc[i][nt][c];
  }
  __syncthreads();

  // ---- reduction: k groups of this CTA, then the Ck CTAs of the cluster ----
  // Work item = (part, tile i, nt, row parity r, lane): columns 2i and 2i+1 of one
  // output row (c = r and c = r + 2), written as one half2.
  constexpr int kItems = kCm * kTiles * NT * 2 * 32;
  const int sum_off = CW * kRegs * 32;  // per-CTA sums after the k-group slots
  if (p.Ck == 1) {
    for (int e = threadIdx.x; e < kItems; e += kThreads) {
      const int ln = e & 31;
      int t = e >> 5;
      const int r = t & 1;
      t >>= 1;
      const int nt = t % NT;
      t /= NT;
      const int i = t % kTiles;
      const int mp = t / kTiles;
      const int n = nt * 8 + 2 * (ln & 3) + r;
      if (n >= p.N) continue;
      const int reg = (i * NT + nt) * 4 + r;
      float lo = 0.0f, hi = 0.0f;
#pragma unroll 4
      for (int g = 0; g < kKG; ++g) {
        const float* sl = slots + (g * kCm + mp) * kRegs * 32 + ln;
        lo += sl[reg * 32];
        hi += sl[(reg + 2) * 32];
      }
      const int col = c0 + mp * 8 * MR + (ln >> 2) * MR + 2 * i;
      store_half2(p.out + static_cast<size_t>(n) * p.M + col, lo, hi);
    }
    return;
  }
  // in-CTA: sum the k groups into this CTA's partial tile
  for (int e = threadIdx.x; e < kCm * kRegs * 32; e += kThreads) {
    const int ln = e & 31, reg = (e >> 5) % kRegs, mp = (e >> 5) / kRegs;
    float v = 0.0f;
#pragma unroll 4
    for (int g = 0; g < kKG; ++g) v += slots[((g * kCm + mp) * kRegs + reg) * 32 + ln];
    slots[sum_off + e] = v;
  }
  cluster_sync();
  {
    const int per = (kItems + p.Ck - 1) / p.Ck;
    const int e0 = q * per, e1 = min(kItems, e0 + per);
    const uint32_t base = smem_u32(slots + sum_off);
    for (int e = e0 + static_cast<int>(threadIdx.x); e < e1; e += kThreads) {
      const int ln = e & 31;
      int t = e >> 5;
      const int r = t & 1;
      t >>= 1;
      const int nt = t % NT;
      t /= NT;
      const int i = t % kTiles;
      const int mp = t / kTiles;
      const int n = nt * 8 + 2 * (ln & 3) + r;
      if (n >= p.N) continue;
      const int il = (mp * kRegs + (i * NT + nt) * 4 + r) * 32 + ln;
      float lo = 0.0f, hi = 0.0f;
      for (int c = 0; c < p.Ck; ++c) {
        const uint32_t a = mapa_shared(base, static_cast<uint32_t>(c));
        lo += ld_shared_cluster_f32(a + 4u * il);
        hi += ld_shared_cluster_f32(a + 4u * (il + 64));
      }
      const int col = c0 + mp * 8 * MR + (ln >> 2) * MR + 2 * i;
      store_half2(p.out + static_cast<size_t>(n) * p.M + col, lo, hi);
    }
  }
  cluster_sync();  // peers may still be reading this CTA's sums
}

// ---------------------------------------------------------------------------
// Stream-K path (M % 256 == 0): one CTA per SM, equal shares of the work.
//
// A work unit is one 16-row slice of one 256-column strip; units are ordered strip
// by strip and CTA c takes units [c U / G, (c + 1) U / G). With exactly one CTA per
// SM no SM ever holds two CTAs of the same call (the next call's CTA, launched early
// through programmatic dependent launch, takes the other half of the SM and
// prefetches its weights). A CTA's units form one or more segments (runs within one
// strip); each segment's partial tile [N][256] goes to its own workspace slot, and
// the CTA that completes a strip (per-strip arrival counter) sums the slots in a
// fixed order and stores fp16: no atomics on data, deterministic results.
// ---------------------------------------------------------------------------
struct SkParams {
  uint16_t* out;        // [N, M] fp16
  const uint16_t* act;  // [N, K] fp16
  uint32_t* err;        // optional device error word
  float* ws;            // partial tiles [strip][slot][N][256] fp32
  uint32_t* cnt;        // per-strip arrival counters, zero between calls
  int N, K, M;
  int KS;               // slices per strip
  int U;                // strips * KS
  int S;                // stages in the ring
  int xoff, xstride;    // activation tile: offset, bytes per batch row
  int redoff;           // k-group reduction tile [kKG][N][256] fp32
  int baroff;
  int maxP;             // workspace slots per strip
  int rpass;            // batch rows per k-group reduction pass (tile = kKG * rpass * 1 KB)
};

// Row stride (floats) of the k-group reduction tile: 256 columns plus one pad float per
// 32, and a stride of 4 (mod 16) between batch rows, so the 32 lanes of a warp park
// their partial sums in 32 distinct banks.
constexpr int kRedRow = 276;

// Dequant of the stream-K kernel: false = exact (the MMA operand is the reference's
// fp16((n - 8) * s)); true = scale folded into the conversion (fewer instructions,
// operand fp16(n * s) plus an exact -8 s correction; about 7e-4 relative error).
constexpr bool kFold = false;

// first CTA whose unit range contains unit x (ranges [c U / G, (c + 1) U / G))
__device__ __forceinline__ int sk_owner(long long x, int G, int U) {
  return static_cast<int>(((x + 1) * G - 1) / U);
}

template <int NT, int MR, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1) k_gemm_sk(const __grid_constant__ WMaps maps, const SkParams p) {
  using L = Layout<256, 1>;
  constexpr int kTiles = MR / 2;
  constexpr int kCm = 256 / (8 * MR);  // column parts (one warp each)
  constexpr int kKG = CW / kCm;        // k groups
  static_assert(kCm * kKG == CW, "warp layout");
  constexpr int kCT = CW * 32;         // consumer threads
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* xs = smem + p.xoff;
  float* red = reinterpret_cast<float*>(smem + p.redoff);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.baroff);
  uint64_t* empty = full + kMaxStages;
  uint32_t* flag = reinterpret_cast<uint32_t*>(empty + kMaxStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
  const int u0 = static_cast<int>(static_cast<long long>(c) * p.U / G);
  const int u1 = static_cast<int>(static_cast<long long>(c + 1) * p.U / G);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, CW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  bool timeout = false;  // after a timed-out wait a thread waits no more
#define MB_WAIT(bar, parity)                                  \
  do {                                                        \
    if (!timeout && !mbar_wait((bar), (parity))) timeout = true; \
  } while (0)

  if (warp == CW) {
    // ---------------- producer: weights only, ahead of the dependency wait ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int st = 0;
      for (int u = u0; u < u1;) {
        const int strip = u / p.KS, ks = u - strip * p.KS;
        const int len = min(u1 - u, p.KS - ks);
        const int ey[1] = {strip}, ex[1] = {0};
        for (int i = 0; i < len; i += kSPS, ++st) {
          const int s = st % p.S;
          if (st >= p.S) MB_WAIT(empty + s, ((st / p.S) - 1) & 1);
          issue_stage<256, 1>(maps, stages + s * L::kStageBytes, full + s, (ks + i) * kSliceRows,
                              min(kSPS, len - i), ey, ex, pol);
        }
        u += len;
      }
    }
  } else {
    // ---------------- consumers ----------------
    const int tid = threadIdx.x;
    const int g4 = lane >> 2, t4 = lane & 3;
    const int mpart = warp % kCm, kg = warp / kCm;
    const int mcol = mpart * 8 * MR + g4 * MR;  // first column of this thread's run
    const int nb = mcol / 2, grp = mcol / 32;

    pdl_wait();  // activations (and the output) belong to the previous kernel until now
    // stage x[n][k] of all this CTA's slices: row n holds local slice l at bytes [32 l, 32 l + 32)
    const int nsl = u1 - u0;
    for (int idx = tid; idx < p.N * nsl * 2; idx += kCT) {
      const int n = idx / (nsl * 2), cc = idx - n * (nsl * 2);
      const int u = u0 + (cc >> 1);
      const int k = (u % p.KS) * kSliceRows + (cc & 1) * 8;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (k < p.K) v = __ldg(reinterpret_cast<const uint4*>(p.act + static_cast<size_t>(n) * p.K + k));
      *reinterpret_cast<uint4*>(xs + n * p.xstride + cc * 16) = v;
    }
    named_bar_sync(1, kCT);
    bool xok[NT];
    const uint8_t* xbase[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nt * 8 + g4;
      xok[nt] = n < p.N;
      xbase[nt] = xs + (xok[nt] ? n : 0) * p.xstride;
    }

    int st = 0, lbase = 0;
    for (int u = u0; u < u1;) {
      const int strip = u / p.KS, ks = u - strip * p.KS;
      const int len = min(u1 - u, p.KS - ks);
      const int nst_seg = (len + kSPS - 1) / kSPS;
      float acc[kTiles][NT][4], corr[NT][4];
#pragma unroll
      for (int i = 0; i < kTiles; ++i)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[i][nt][q] = 0.0f;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 4; ++q) corr[nt][q] = 0.0f;

      // This warp's slice of each stage of the segment is slice kg (eight k groups, eight
      // slices per full stage); the last stage may be partial. Double-buffered in
      // registers: wait for the next stage, load its slice, then compute the current one,
      // so the shared-memory latency hides behind the arithmetic.
      static_assert(kKG == kSPS, "one slice per warp per stage");
      const int nlast = len - (nst_seg - 1) * kSPS;
      const int nmine = (kg < nlast) ? nst_seg : nst_seg - 1;
      // One slice per stage for this warp; ring slot and phase advance incrementally (no
      // division in the loop).
      int ls = st % p.S;              // ring slot of segment stage 0
      uint32_t lph = (st / p.S) & 1;  // its phase
      for (int t = 0; t < nmine; ++t) {
        if (!timeout && !mbar_wait(full + ls, lph)) timeout = true;
        const uint8_t* xr[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) xr[nt] = xbase[nt] + (lbase + t * kSPS + kg) * 32;
        consume_slice<NT, 256, 1, MR>(stages + ls * L::kStageBytes, kg * kSliceRows + 2 * t4, nb, grp, grp, xr, xok,
                                      t4, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + ls);
        if (++ls == p.S) {
          ls = 0;
          lph ^= 1u;
        }
      }
      if (nmine < nst_seg) {  // no slice for this warp in the partial last stage: release it
        // after its full barrier, so this arrival cannot count toward the slot's previous use
        if (!timeout && !mbar_wait(full + ls, lph)) timeout = true;
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + ls);
      }
      st += nst_seg;

      // ---- segment epilogue: k groups -> one partial tile -> workspace / output ----
      // accumulator (i, nt, q) of this thread: batch row 8 nt + 2 t4 + (q & 1), column
      // mcol + 2 i + (q >> 1); the folded dequant leaves + 8 s per weight: subtract 8 corr
      const long long sx0 = static_cast<long long>(strip) * p.KS;
      const int cf = sk_owner(sx0, G, p.U), cl = sk_owner(sx0 + p.KS - 1, G, p.U);
      const int piece = c - cf, npieces = cl - cf + 1;
      uint16_t* ob = p.out + static_cast<size_t>(strip) * 256;
      float* wsl = p.ws + static_cast<size_t>(strip) * p.maxP * p.N * 256;
      for (int n0 = 0; n0 < p.N; n0 += p.rpass) {  // batch rows in passes that fit the tile
        const int nr = min(p.rpass, p.N - n0);
#pragma unroll
        for (int i = 0; i < kTiles; ++i)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int n = nt * 8 + 2 * t4 + (q & 1) - n0;
              const int col = mcol + 2 * i + (q >> 1);
              if (n >= 0 && n < nr)
                red[(kg * nr + n) * kRedRow + col + (col >> 5)] =
                    kFold ? fmaf(-8.0f, corr[nt][q], acc[i][nt][q]) : acc[i][nt][q];
            }
        named_bar_sync(1, kCT);
        for (int e = tid; e < nr * 128; e += kCT) {
          const int n = e >> 7, col = (e & 127) * 2;
          float lo = 0.0f, hi = 0.0f;
#pragma unroll
          for (int g = 0; g < kKG; ++g) {
            const float* rr = red + (g * nr + n) * kRedRow + col + (col >> 5);
            lo += rr[0];
            hi += rr[1];
          }
          if (npieces == 1) {
            store_half2(ob + static_cast<size_t>(n0 + n) * p.M + col, lo, hi);
          } else {
            *reinterpret_cast<float2*>(wsl + (static_cast<size_t>(piece) * p.N + n0 + n) * 256 + col) =
                make_float2(lo, hi);
          }
        }
        named_bar_sync(1, kCT);  // the tile is free for the next pass
      }
      if (npieces > 1) {
        __threadfence();  // this slot is visible before the arrival is counted
        named_bar_sync(1, kCT);
        if (tid == 0) flag[0] = (atomicAdd(p.cnt + strip, 1u) == static_cast<uint32_t>(npieces - 1)) ? 1u : 0u;
        named_bar_sync(1, kCT);
        if (flag[0]) {
          __threadfence();
          for (int e = tid; e < p.N * 128; e += kCT) {
            const int n = e >> 7, col = (e & 127) * 2;
            const float* src = wsl + static_cast<size_t>(n) * 256 + col;
            const size_t pstride = static_cast<size_t>(p.N) * 256;
            float lo = 0.0f, hi = 0.0f;
            for (int pc0 = 0; pc0 < npieces; pc0 += 8) {  // eight loads in flight, summed in order
              float2 v[8];
#pragma unroll
              for (int k = 0; k < 8; ++k)
                if (pc0 + k < npieces) v[k] = __ldcg(reinterpret_cast<const float2*>(src + (pc0 + k) * pstride));
#pragma unroll
              for (int k = 0; k < 8; ++k)
                if (pc0 + k < npieces) {
                  lo += v[k].x;
                  hi += v[k].y;
                }
            }
            store_half2(ob + static_cast<size_t>(n) * p.M + col, lo, hi);
          }
          if (tid == 0) p.cnt[strip] = 0u;  // ready for the next call
        }
        named_bar_sync(1, kCT);
      }
      lbase += len;
      u += len;
    }
  }
#undef MB_WAIT
  if (timeout && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// Generic path (any M with K*M % 256 == 0, any K): one thread per output column,
// flat super-block indexing as in fused_batched_gemm_int4 (batched_gemm.metal:146-155),
// activations staged in shared memory. Correct for every shape; the TMA path above
// is the fast one.
// ---------------------------------------------------------------------------
template <int NB>
__global__ void __launch_bounds__(128) k_gemm_generic(const uint16_t* __restrict__ act, const uint8_t* __restrict__ sb,
                                                      uint16_t* __restrict__ out, int N, int K, int M) {
  constexpr int KC = 64;
  __shared__ float xsm[NB][KC];
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  float acc[NB];
#pragma unroll
  for (int n = 0; n < NB; ++n) acc[n] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += KC) {
    __syncthreads();
    for (int t = threadIdx.x; t < NB * KC; t += blockDim.x) {
      const int n = t / KC, kk = t % KC;
      xsm[n][kk] = (n < N && k0 + kk < K) ? __half2float(__ushort_as_half(act[static_cast<size_t>(n) * K + k0 + kk]))
                                          : 0.0f;
    }
    __syncthreads();
    if (m < M) {
      const int kend = min(KC, K - k0);
      for (int kk = 0; kk < kend; ++kk) {
        const long long flat = static_cast<long long>(k0 + kk) * M + m;
        const uint8_t* b = sb + (flat >> 8) * kSB;
        const int e = static_cast<int>(flat & 255);
        const int byte = __ldg(b + 16 + (e >> 1));
        const int qv = ((e & 1) ? (byte >> 4) : (byte & 15)) - 8;
        const __half s = __ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(b) + (e >> 5)));
        const float w = __half2float(__hmul(__int2half_rn(qv), s));
#pragma unroll
        for (int n = 0; n < NB; ++n) acc[n] = fmaf(xsm[n][kk], w, acc[n]);
      }
    }
  }
  if (m < M)
#pragma unroll
    for (int n = 0; n < NB; ++n)
      if (n < N) out[static_cast<size_t>(n) * M + m] = __half_as_ushort(__float2half_rn(acc[n]));
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct Plan {
  int ws = 0, P = 1, Ck = 1, nt = 1, S = 0, smem = 0, xstride = 0, xbytes = 0, ctas = 0;
  bool fast = false;
};

static constexpr int kCW = 8;                   // consumer warps per CTA
static constexpr int kSmemBudget = 112 * 1024;  // half an SM: room for the next call's CTA

static int stage_bytes_of(int ws, int P) {
  if (ws == 256) return Layout<256, 1>::kStageBytes;
  return P == 1 ? Layout<128, 1>::kStageBytes : Layout<128, 2>::kStageBytes;
}

// bytes of the final-reduction scratch (k-group slots + per-CTA sums), which reuses
// the stage ring and the activation slice
static int reduce_bytes(int nt, int ws) {
  const int mr = std::min(32 / nt, ws / 8);
  const int regs = (mr / 2) * nt * 4;
  const int cm = ws / (8 * mr);
  return (kCW + cm) * regs * 32 * 4;
}

// Picks the strip width, K split (cluster size) and ring depth for a shape: the most
// CTAs that fit one wave of the SMs (all SMs stream the weights), then no cluster
// (no cross-CTA reduction), then the wider strip (activations read fewer times).
static Plan plan_gemm(int N, int K, int M, int sms) {
  Plan pl;
  pl.nt = N <= 8 ? 1 : (N <= 16 ? 2 : 4);
  if (K % 8 != 0 || M % 128 != 0) return pl;
  const int P = (M % 256 == 0) ? 1 : ((M % 128 == 0) ? 2 : 0);
  if (P == 0) return pl;
  const int KS = (K + kSliceRows - 1) / kSliceRows;
  long long best_key = -1;
  for (int ws : {256, 128}) {
    if (ws == 256 && P != 1) continue;
    const int strips = M / ws;
    for (int ck = 1; ck <= kMaxCk && ck <= KS; ++ck) {
      const long long ctas = static_cast<long long>(strips) * ck;
      if (ck > 1 && ctas > sms) break;
      const int slices = (KS + ck - 1) / ck;
      const int xstride = slices * kSliceRows * 2 + 16;
      const int xbytes = (N * xstride + 127) / 128 * 128;
      if (xbytes + 2 * stage_bytes_of(ws, P) + 2048 > kSmemBudget) continue;
      const long long used = std::min<long long>(ctas, sms);
      // one wave: more SMs first (quantised to 1/16 of the SMs), then wider strips
      // (wider per-thread runs: fewer instructions per weight), then fewer CTAs per
      // cluster
      const long long key = (used * 16 / sms) * 1000 + ws / 64 * 10 + (8 - ck);
      if (key > best_key) {
        best_key = key;
        pl.ws = ws;
        pl.Ck = ck;
        pl.xstride = xstride;
        pl.xbytes = xbytes;
        pl.ctas = static_cast<int>(ctas);
      }
    }
  }
  if (best_key < 0) return pl;
  pl.P = P;
  const int sb = stage_bytes_of(pl.ws, P);
  const int KSc = (KS + pl.Ck - 1) / pl.Ck;
  const int need = (KSc + kSPS - 1) / kSPS;  // stages that hold the CTA's whole slice
  int S = (kSmemBudget - 2048 - pl.xbytes) / sb;
  S = std::max(2, std::min(std::min(S, kMaxStages), need));
  // the reduction scratch lives in the stage ring followed by the activation slice
  while (S * sb + pl.xbytes < reduce_bytes(pl.nt, pl.ws) && S < kMaxStages) ++S;
  if (S * sb + pl.xbytes < reduce_bytes(pl.nt, pl.ws)) pl.xbytes = reduce_bytes(pl.nt, pl.ws) - S * sb;
  pl.S = S;
  // at least 116 KB: one CTA per SM, so two CTAs of one call never share an SM
  pl.smem = std::max(116 * 1024, 1024 + S * sb + pl.xbytes + 2 * kMaxStages * 8);
  pl.fast = true;
  return pl;
}

template <int NT, int WS, int P>
static int launch_fast(const Plan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
                       uint32_t* err, cudaStream_t st) {
  using L = Layout<WS, P>;
  auto kern = k_gemm_int4<NT, WS, P, kCW>;
  static bool attr_set[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MB_ERR_LAUNCH;
  if (!attr_set[dev]) {
    // full shared-memory carveout, so two ~112 KB CTAs (this call and the next) fit an SM
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return MB_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  WMaps maps;
  // 3-D view of the stream: [144 bytes][super-blocks per period][periods of P rows]
  const uint64_t sbp = static_cast<uint64_t>(P) * M / 256;
  const uint64_t dims[3] = {kSB, sbp, static_cast<uint64_t>(K / P)};
  const uint64_t strides[2] = {kSB, sbp * kSB};
  bool ok;
  if (WS == 256) {
    const uint32_t bf[3] = {kSB, 1, kStageRows}, bs[3] = {kSB, 1, kSliceRows};
    ok = encode_tmap_3d_u8(&maps.full_a, sb, dims, strides, bf) &&
         encode_tmap_3d_u8(&maps.slice_a, sb, dims, strides, bs);
    maps.full_b = maps.full_a;
    maps.slice_b = maps.slice_a;
  } else {
    const uint32_t sf[3] = {16, 1, kStageRows / P}, ss[3] = {16, 1, kSliceRows / P};
    const uint32_t nf[3] = {L::kNibRow, 1, kStageRows / P}, ns[3] = {L::kNibRow, 1, kSliceRows / P};
    ok = encode_tmap_3d_u8(&maps.full_a, sb, dims, strides, sf) &&
         encode_tmap_3d_u8(&maps.slice_a, sb, dims, strides, ss) &&
         encode_tmap_3d_u8(&maps.full_b, sb, dims, strides, nf) &&
         encode_tmap_3d_u8(&maps.slice_b, sb, dims, strides, ns);
  }
  if (!ok) return MB_ERR_LAUNCH;
  GemmParams prm;
  prm.out = out;
  prm.act = act;
  prm.err = err;
  prm.N = N;
  prm.K = K;
  prm.M = M;
  prm.KS = (K + kSliceRows - 1) / kSliceRows;
  prm.Ck = pl.Ck;
  prm.S = pl.S;
  prm.xstride = pl.xstride;
  prm.xbytes = pl.xbytes;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((M / WS) * pl.Ck);
  cfg.blockDim = dim3((kCW + 1) * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = pl.Ck;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, maps, prm) != cudaSuccess) return MB_ERR_LAUNCH;
  return launch_status();
}

template <int NT>
static int dispatch_fast(const Plan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
                         uint32_t* err, cudaStream_t st) {
  if (pl.ws == 256) return launch_fast<NT, 256, 1>(pl, act, sb, out, N, K, M, err, st);
  if (pl.ws == 128)
    return pl.P == 1 ? launch_fast<NT, 128, 1>(pl, act, sb, out, N, K, M, err, st)
                     : launch_fast<NT, 128, 2>(pl, act, sb, out, N, K, M, err, st);
  return MB_ERR_UNSUPPORTED;
}

static int launch_generic(const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M, cudaStream_t st) {
  const dim3 grid((M + 127) / 128);
  if (N <= 8)
    k_gemm_generic<8><<<grid, 128, 0, st>>>(act, sb, out, N, K, M);
  else if (N <= 16)
    k_gemm_generic<16><<<grid, 128, 0, st>>>(act, sb, out, N, K, M);
  else
    k_gemm_generic<32><<<grid, 128, 0, st>>>(act, sb, out, N, K, M);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Stream-K host side
// ---------------------------------------------------------------------------
struct SkPlan {
  bool ok = false;
  int nt = 1, mr = 32, G = 0, S = 0, smem = 0, xoff = 0, xstride = 0, redoff = 0, baroff = 0, maxP = 0, rpass = 1;
  size_t ws_bytes = 0;  // workspace: counters then partial tiles
};
static constexpr int kSkCW = 8;
// One CTA per SM (more than half an SM's shared memory): the grid is exactly one wave,
// no SM runs two CTAs of a call, and each CTA has the whole register file.
static constexpr int kSkSmem = 220 * 1024;

static SkPlan plan_sk(int N, int K, int M, int sms) {
  SkPlan pl;
  if (N < 1 || N > 8 || K % 8 != 0 || M % 256 != 0) return pl;
  pl.nt = 1;
  pl.mr = 32;
  const int strips = M / 256, KS = (K + kSliceRows - 1) / kSliceRows;
  const long long U = static_cast<long long>(strips) * KS;
  if (U > (1LL << 30)) return pl;
  pl.G = static_cast<int>(std::min<long long>(sms, U));
  const int nsl = static_cast<int>((U + pl.G - 1) / pl.G);  // most slices of any CTA
  const int kKG = kSkCW / (256 / (8 * pl.mr));
  pl.xstride = nsl * 32 + 16;
  const int xbytes = (N * pl.xstride + 127) / 128 * 128;
  pl.rpass = N;  // one pass: the reduction tile is kKG x N x 1 KB
  const int redbytes = kKG * pl.rpass * kRedRow * 4;
  const int sb = Layout<256, 1>::kStageBytes;
  const int need = (nsl + kSPS - 1) / kSPS + 1;  // a run may straddle two strips
  int S = (kSkSmem - 1024 - 256 - xbytes - redbytes) / sb;
  S = std::min(std::min(S, kMaxStages), need);
  if (S < 2) return pl;
  pl.S = S;
  pl.xoff = S * sb;
  pl.redoff = pl.xoff + xbytes;
  pl.baroff = pl.redoff + redbytes;
  pl.smem = std::max(116 * 1024, 1024 + pl.baroff + 2 * kMaxStages * 8 + 16);
  // slots per strip: CTAs touching one strip
  const long long per = U / pl.G;  // every CTA has at least this many units
  pl.maxP = static_cast<int>(std::min<long long>(pl.G, KS / std::max<long long>(per, 1) + 2));
  pl.ws_bytes = static_cast<size_t>(strips) * 4 + 256 +
                static_cast<size_t>(strips) * pl.maxP * N * 256 * sizeof(float);
  pl.ok = true;
  return pl;
}

template <int NT>
static int launch_sk(const SkPlan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
                     void* ws, uint32_t* err, cudaStream_t st) {
  auto kern = k_gemm_sk<NT, 32 / NT, kSkCW>;
  static bool attr_set[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MB_ERR_LAUNCH;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return MB_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  WMaps maps;
  const uint64_t dims[3] = {kSB, static_cast<uint64_t>(M / 256), static_cast<uint64_t>(K)};
  const uint64_t strides[2] = {kSB, static_cast<uint64_t>(M / 256) * kSB};
  const uint32_t bf[3] = {kSB, 1, kStageRows}, bs[3] = {kSB, 1, kSliceRows};
  if (!encode_tmap_3d_u8(&maps.full_a, sb, dims, strides, bf) || !encode_tmap_3d_u8(&maps.slice_a, sb, dims, strides, bs))
    return MB_ERR_LAUNCH;
  maps.full_b = maps.full_a;
  maps.slice_b = maps.slice_a;
  const int strips = M / 256;
  SkParams prm;
  prm.out = out;
  prm.act = act;
  prm.err = err;
  prm.cnt = static_cast<uint32_t*>(ws);
  prm.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + (static_cast<size_t>(strips) * 4 + 255) / 256 * 256);
  prm.N = N;
  prm.K = K;
  prm.M = M;
  prm.KS = (K + kSliceRows - 1) / kSliceRows;
  prm.U = strips * prm.KS;
  prm.S = pl.S;
  prm.xoff = pl.xoff;
  prm.xstride = pl.xstride;
  prm.redoff = pl.redoff;
  prm.baroff = pl.baroff;
  prm.maxP = pl.maxP;
  prm.rpass = pl.rpass;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.G);
  cfg.blockDim = dim3((kSkCW + 1) * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, maps, prm) != cudaSuccess) return MB_ERR_LAUNCH;
  return launch_status();
}

// One launch over up to 32 batch rows. Stream-K (needs the workspace) up to 16 rows,
// the tensor-core path up to 32, else the cluster kernel or the generic one.
static int gemm_rows(const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M, void* ws,
                     size_t ws_bytes, uint32_t* err, cudaStream_t st) {
  if (aligned(act, 16) && aligned(sb, 16) && aligned(out, 4)) {
    if (ws != nullptr && aligned(ws, 256)) {
      const SkPlan sp = plan_sk(N, K, M, sm_count());
      if (sp.ok && ws_bytes >= sp.ws_bytes) return launch_sk<1>(sp, act, sb, out, N, K, M, ws, err, st);
    }
    tc::TcPlan tp;
    if (N > 16 && tc::plan(N, K, M, sm_count(), &tp)) return tc::launch(tp, act, sb, out, N, K, M, err, st);
    const Plan pl = plan_gemm(N, K, M, sm_count());
    if (pl.fast) {
      if (pl.nt == 1) return dispatch_fast<1>(pl, act, sb, out, N, K, M, err, st);
      if (pl.nt == 2) return dispatch_fast<2>(pl, act, sb, out, N, K, M, err, st);
      return dispatch_fast<4>(pl, act, sb, out, N, K, M, err, st);
    }
  }
  return launch_generic(act, sb, out, N, K, M, st);
}

static int gemm_all(const uint16_t* act, const uint8_t* sb, uint16_t* out, int32_t N, int32_t K, int32_t M, void* ws,
                    size_t ws_bytes, uint32_t* dev_err, void* stream) {
  if (N < 1 || K < 1 || M < 1 || (static_cast<int64_t>(K) * M) % 256 != 0) return MB_ERR_ARGS;
  if (!act || !sb || !out) return MB_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int r0 = 0; r0 < N; r0 += 32) {
    const int nb = std::min(32, N - r0);
    const int rc = gemm_rows(act + static_cast<size_t>(r0) * K, sb, out + static_cast<size_t>(r0) * M, nb, K, M, ws,
                             ws_bytes, dev_err, st);
    if (rc != MB_OK) return rc;
  }
  return MB_OK;
}

}  // namespace mb

using namespace mb;

extern "C" {

int32_t mb_int4_gemm(const uint16_t* act, const uint8_t* sb, uint16_t* out, int32_t N, int32_t K, int32_t M,
                     uint32_t* dev_err, void* stream) {
  return gemm_all(act, sb, out, N, K, M, nullptr, 0, dev_err, stream);
}

size_t mb_int4_gemm_workspace_size(int32_t N, int32_t K, int32_t M) {
  if (N < 1 || K < 1 || M < 1) return 0;
  const SkPlan sp = plan_sk(std::min(N, 8), K, M, sm_count());
  return sp.ok ? sp.ws_bytes : 0;
}

int32_t mb_int4_gemm_ws(const uint16_t* act, const uint8_t* sb, uint16_t* out, int32_t N, int32_t K, int32_t M,
                        void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream) {
  if (workspace != nullptr && !aligned(workspace, 256)) return MB_ERR_ALIGN;
  return gemm_all(act, sb, out, N, K, M, workspace, workspace_bytes, dev_err, stream);
}

int32_t mb_int4_gemm_plan(int32_t N, int32_t K, int32_t M, int32_t* info) {
  if (!info) return MB_ERR_NULL;
  if (N < 1 || K < 1 || M < 1) return MB_ERR_ARGS;
  const SkPlan sp = plan_sk(std::min(N, 32), K, M, sm_count());  // N <= 8 only
  if (sp.ok) {  // stream-K path (with a workspace)
    info[0] = 3;
    info[1] = 256;
    info[2] = 1;
    info[3] = sp.G;
    info[4] = sp.S;
    info[5] = sp.smem;
    info[6] = sp.maxP;
    info[7] = sp.nt;
    return MB_OK;
  }
  tc::TcPlan tp;
  if (std::min(N, 32) > 16 && tc::plan(std::min(N, 32), K, M, sm_count(), &tp)) {  // tensor-core path
    info[0] = 2;
    info[1] = 256;
    info[2] = tp.Ck;
    info[3] = tp.ctas;
    info[4] = tp.S;
    info[5] = tp.smem;
    info[6] = tp.tcols;
    info[7] = tp.NP;
    return MB_OK;
  }
  const Plan pl = plan_gemm(std::min(N, 32), K, M, sm_count());
  info[0] = pl.fast ? 1 : 0;
  info[1] = pl.ws;
  info[2] = pl.Ck;
  info[3] = pl.fast ? pl.ctas : (M + 127) / 128;
  info[4] = pl.S;
  info[5] = pl.smem;
  info[6] = pl.P;
  info[7] = pl.nt;
  return MB_OK;
}

}  // extern "C"
