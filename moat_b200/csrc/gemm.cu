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
//    columns. Each strip is handled by one thread-block cluster of Ck CTAs that split
//    its K rows; the grid (strips x Ck) is one wave of the SMs, one CTA per SM.
//  * One producer warp per CTA streams the CTA's super-block rows with 3-D TMA tile
//    loads (cp.async.bulk.tensor, L2 evict-first, no multicast) into a ring of
//    shared-memory stages guarded by mbarriers, and re-lays each landed stage's fp16
//    group scales as (row pair, group) words for the consumers. Weights never depend on
//    the previous kernel, so the producer starts before griddepcontrol.wait
//    (programmatic dependent launch) and the ring fills while the previous grid ends.
//  * Each scale group (32 columns) of the strip has kKG consumer warps (16 warps per
//    CTA). ldmatrix.trans of the group's nibble rows gives each lane two bytes of two
//    consecutive k rows in one register, which a lop3 with the fp16 magic exponent
//    turns into an mma.m16n8k16 A fragment pair (k, k+1) without any byte permute:
//    exact integers q = n - 8. Every row of an m16 tile lies in one scale group, so the
//    group scale of row k is applied to the activations instead (B' = fp16(x[n, k] *
//    s[k, g]), two f16x2 multiplies per 16 k rows and 8 batch rows) and the tensor core
//    sums q * B' in fp32. The kKG warps of a group take alternate stages (one batch
//    tile) or alternate slices of every stage (more tiles, or few stages).
//  * Reduction: every warp stores its partial tile straight into the shared memory of
//    the cluster CTA that owns those columns (st.shared::cluster), one cluster barrier,
//    and each owner adds the Ck x kKG partials of its columns in a fixed order:
//    deterministic, no global workspace, no atomics.
#include <algorithm>
#include <type_traits>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "peer_ll.cuh"

namespace mb {

constexpr int kSB = 144;        // bytes per super-block
constexpr int kSliceRows = 16;  // k rows per MMA slice
constexpr int kSPS = 8;         // slices per full stage (128 rows)
constexpr int kStageRows = kSPS * kSliceRows;
constexpr int kMaxStages = 8;
constexpr int kMaxCk = 8;
constexpr int kAhead = 3;  // weight stages in flight per CTA while the ring first fills
constexpr int kCW = 16;    // consumer warps per CTA (two or four per scale group)

// Shared-memory layout of one pipeline stage (128 rows of the CTA's strip).
//  WS = 256: full 144-byte super-block rows (scales then nibbles), row stride 144 B.
//  WS = 128: a 16-byte scale row per k row, then the strip's 64 nibble bytes in a row
//  padded to 80 bytes by the TMA box. With P = 2 row phases (M % 256 == 128) the rows
//  of each phase are stored together.
// Row strides of 144 and 80 bytes put 8 consecutive rows of a region in 8 distinct
// 16-byte bank groups, so every ldmatrix below is conflict free. For P = 2 the 16 k
// rows of a slice are read as 8 even rows (one region) then 8 odd rows, which is also
// the order in which the slice's activations are staged.
template <int WS, int P>
struct Layout {
  static_assert(WS == 256 || WS == 128, "strip width");
  static_assert(WS != 256 || P == 1, "a 256-wide strip needs M % 256 == 0");
  static_assert(P == 1 || P == 2, "row phases");
  static constexpr int kGS = WS / 32;  // scale groups per strip row
  static constexpr int kNibRow = 80;
  static constexpr int kScRegion = kStageRows * 16;
  static constexpr int kStageBytes = (WS == 256) ? kStageRows * kSB : kStageRows * (16 + kNibRow);
  static constexpr int kRowsPerPhase = kStageRows / P;
  static constexpr int kScBytes = kSPS * kGS * 4 * 8;  // re-laid scale pairs of one stage
  static __device__ __host__ constexpr int bytes(int n) {  // tx bytes of a stage with n slices
    return (WS == 256) ? n * kSliceRows * kSB : n * kSliceRows * (16 + kNibRow);
  }
  // byte offset of row k's scale chunk / first strip nibble byte within a stage
  static __device__ __host__ constexpr int sc(int k) {
    return (WS == 256) ? k * kSB : ((k & (P - 1)) * kRowsPerPhase + k / P) * 16;
  }
  static __device__ __host__ constexpr int nib(int k) {
    return (WS == 256) ? k * kSB + 16 : kScRegion + ((k & (P - 1)) * kRowsPerPhase + k / P) * kNibRow;
  }
  // stage row of MMA k index i (0..15) of slice sl
  static __device__ __host__ constexpr int row_of(int sl, int i) {
    return P == 1 ? kSliceRows * sl + i : kSliceRows * sl + (i < 8 ? 2 * i : 2 * (i - 8) + 1);
  }
  static constexpr int kSliceStride = nib(kSliceRows) - nib(0);  // nibble bytes between slices
  static constexpr int kScSliceStride = sc(kSliceRows) - sc(0);
};

struct GemmParams {
  uint16_t* out;        // [N, M] fp16
  const uint16_t* act;  // [N, K] fp16
  uint32_t* err;        // optional device error word (may be null)
  int N, K, M;
  int KS;               // k slices (ceil(K / 16))
  int Ck;               // CTAs per cluster = K split
  int S;                // stages in the ring
  int xcstride;         // bytes per 128-k chunk of activations (N rows of kXRow bytes, 128-aligned)
  int scboff;           // byte offset of the re-laid scale pairs [S][kScBytes]
  int xoff;             // byte offset of the activation chunks
  int recvoff;          // byte offset of the receive slots [Ck][kKG][N][rp] floats
  int baroff;           // byte offset of the mbarriers
  int rp;               // floats per receive row (owned columns + 4 pad)
  int sl_first[kMaxCk + 1];  // k slices [sl_first[q], sl_first[q + 1]) go to CTA q of a cluster
  int gfirst[kMaxCk + 1];    // CTA q owns strip groups [gfirst[q], gfirst[q + 1])
  int owner[8];              // the CTA that owns strip group g
  int split;                 // 1: the kKG warps of a group take alternate stages (all 8 slices each);
                             // 0: they take alternate slices of every stage
  // Row-parallel exchange (XCH kernels only): instead of writing out, the owners store
  // their fp16 rows as low-latency words into slot [epoch parity][xrank] of every
  // rank's exchange buffer (layout in peer_ll.cuh; M is the join's row width D).
  uint8_t* xbuf[kPeerMaxRanks];
  const uint32_t* xstate;  // the join channel's row epochs: this call's epoch is state[row] + 1
  long long xslot;         // fp16 elements of one exchange slot
  int xworld, xrank, xrow0;  // xrow0: exchange row of this launch's first batch row
};

// Activations in shared memory: chunks of 128 k values (one stage) by N rows; a row
// takes 272 bytes (128 values + 8 pad), so consecutive rows start 4 banks apart and
// the B-fragment loads are conflict free.
constexpr int kXRow = 272;

struct WMaps {  // weight tensor maps: full-stage and 16-row boxes (scale / nibble rows)
  CUtensorMap full_a, full_b, slice_a, slice_b;
};

// Shared-memory loads by 32-bit shared-window address, so the loop's address arithmetic
// stays in 32-bit registers with constant offsets.
__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 ld_shared_v2(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
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

// Producer warp: the landed stage's scales -> [slice][group][t4] words of two half2
// pairs: (s[row(2 t4)], s[row(2 t4 + 1)]) and (s[row(2 t4 + 8)], s[row(2 t4 + 9)]) of
// the strip's group, the pairs a consumer lane multiplies its B fragments by.
// ldmatrix.trans of 8 scale rows gives lane (g4, t4) the scales of super-block group g4
// of rows (2 t4, 2 t4 + 1); grp_m is the first super-block group of the strip in rows
// of MMA half m (the row phase for P = 2).
template <int WS, int P>
__device__ __forceinline__ void relay_scales(const uint8_t* stage, uint8_t* scs, int lane, int grp0, int grp1) {
  using L = Layout<WS, P>;
  constexpr int GS = L::kGS;
  const int g4 = lane >> 2, t4 = lane & 3;
  const int mm = lane >> 3, j8 = lane & 7;
  // matrix mm of an x4: slice 2 pr + (mm >> 1), MMA half m = mm & 1, row j8 of that half
  const uint32_t a0 = smem_u32(stage) + L::sc(L::row_of(mm >> 1, 8 * (mm & 1) + j8));
#pragma unroll
  for (int pr = 0; pr < kSPS / 2; ++pr) {
    uint32_t r[4];
    ldsm_x4_trans(a0 + 2 * pr * L::kScSliceStride, r[0], r[1], r[2], r[3]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int sl = 2 * pr + (i >> 1), m = i & 1;
      const int gl = g4 - (m ? grp1 : grp0);
      if (gl >= 0 && gl < GS)
        *reinterpret_cast<uint32_t*>(scs + ((sl * GS + gl) * 4 + t4) * 8 + 4 * m) = r[i];
    }
  }
}

// The nibble -> fp16 constants of the dequant loop, held in registers for the whole
// kernel (made opaque to the compiler once, so they are not re-created at every use).
struct NibConst {
  uint32_t lo_mask, hi_mask, magic, sub_lo, mul_hi, add_hi;
  __device__ __forceinline__ NibConst()
      : lo_mask(0x000F000Fu), hi_mask(0x00F000F0u), magic(0x64006400u), sub_lo(0x64086408u), mul_hi(0x2C002C00u),
        add_hi(0xD480D480u) {
    asm volatile("" : "+r"(lo_mask), "+r"(hi_mask), "+r"(magic), "+r"(sub_lo), "+r"(mul_hi), "+r"(add_hi));
  }
};

// nibbles_to_half2 with the constants in registers: low nibbles of bytes 0 / 2 of p ->
// (n0 - 8, n2 - 8), high nibbles -> (h0 - 8, h2 - 8), exact.
__device__ __forceinline__ void nib2h(const NibConst& c, uint32_t p, uint32_t& lo, uint32_t& hi) {
  const uint32_t l = lop3<0xEA>(p, c.lo_mask, c.magic);
  const uint32_t h = lop3<0xEA>(p, c.hi_mask, c.magic);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(l), "r"(c.sub_lo));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(hi) : "r"(h), "r"(c.mul_hi), "r"(c.add_hi));
}

__device__ __forceinline__ void store_half4(uint16_t* dst, float a, float b, float c, float d) {
  const __half2 x = __floats2half2_rn(a, b), y = __floats2half2_rn(c, d);
  uint2 v;
  v.x = *reinterpret_cast<const uint32_t*>(&x);
  v.y = *reinterpret_cast<const uint32_t*>(&y);
  *reinterpret_cast<uint2*>(dst) = v;
}

// One 16-row slice of this warp's group (xr: the lane's activation words of the slice,
// k indices 2 t4 and 2 t4 + 8 at +0 / +16): r0 / r1 are lane (g4, t4)'s ldmatrix words of
// MMA k halves 0 / 1 (bytes 2 g4, 2 g4 + 1 of rows 2 t4, 2 t4 + 1 of the half). Tile 0
// maps fragment row g4 to group column 4 g4 and row g4 + 8 to column 4 g4 + 1 (low /
// high nibble of byte 2 g4); tile 1 takes columns 4 g4 + 2 and 4 g4 + 3 (byte 2 g4 + 1).
template <int NT>
__device__ __forceinline__ void consume_slice(const NibConst& kc, uint32_t r0, uint32_t r1, const uint32_t (&xr)[NT],
                                              uint2 sc, float (&acc)[2][NT][4]) {
  uint32_t bp[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint32_t b0 = ld_shared_u32(xr[nt]);
    const uint32_t b1 = ld_shared_u32(xr[nt] + 16);
    bp[nt][0] = hmul2(b0, sc.x);
    bp[nt][1] = hmul2(b1, sc.y);
  }
  uint32_t a0, a1, a2, a3, c0, c1, c2, c3;
  nib2h(kc, r0, a0, a1);
  nib2h(kc, r1, a2, a3);
  nib2h(kc, r0 >> 8, c0, c1);
  nib2h(kc, r1 >> 8, c2, c3);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    mma_16816(acc[0][nt], a0, a1, a2, a3, bp[nt][0], bp[nt][1]);
    mma_16816(acc[1][nt], c0, c1, c2, c3, bp[nt][0], bp[nt][1]);
  }
}

// NT: n-tiles of 8 batch rows (1, 2, 4); WS: strip width; P: row phases (1, 2);
// XCH: the epilogue stores into the exchange buffers instead of out.
// One CTA per SM (16 consumer warps take the SM's registers).
template <int NT, int WS, int P, bool XCH>
__global__ void __launch_bounds__((kCW + 1) * 32, 1)
    k_gemm_int4(const __grid_constant__ WMaps maps, const GemmParams p) {
  using L = Layout<WS, P>;
  constexpr int GS = L::kGS;
  constexpr int kKG = kCW / GS;  // warps per group (k groups): 2 for WS = 256, 4 for WS = 128
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base, derived from the shared array itself so that every access
  // below compiles to a shared-memory (not generic) load or store
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stages = smem;
  uint8_t* scb = smem + p.scboff;
  uint8_t* xs = smem + p.xoff;
  float* recv = reinterpret_cast<float*>(smem + p.recvoff);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.baroff);
  uint64_t* empty = full + kMaxStages;
  uint64_t* ready = empty + kMaxStages;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int strip = blockIdx.x / p.Ck;
  const int q = blockIdx.x - strip * p.Ck;  // == rank in the cluster (cluster dims = (Ck,1,1))
  const int sl0 = p.sl_first[q], sl1 = p.sl_first[q + 1];
  const int nst = (sl1 - sl0 + kSPS - 1) / kSPS;
  const int c0 = strip * WS;
  // per row phase: super-block index within a period (y), first nibble byte of the
  // strip in that super-block (x) and the super-block group of the strip's first column
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
      mbar_init(empty + s, p.split ? GS : kCW);  // the warps that read the stage
      mbar_init(ready + s, 32);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // phase 0 of the cluster barrier: every CTA of the cluster has started (awaited
  // before the first store into a peer's shared memory)
  if (p.Ck > 1) cluster_arrive_relaxed();
  pdl_launch_dependents();

  if (warp == kCW) {
    // ---------------- producer ----------------
    // weights never depend on the previous grid: no griddepcontrol.wait here, so the
    // ring fills (and its scales are re-laid) while the previous grid finishes
    const uint64_t pol = policy_evict_first();
    const int fill = min(p.S, nst);
    int issued = 0, tr = 0;
    auto relay = [&](int st) {
      const int s = st % p.S;
      if (!mbar_wait(full + s, (st / p.S) & 1) && lane == 0 && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
      relay_scales<WS, P>(stages + s * L::kStageBytes, scb + s * L::kScBytes, lane, grp[0], grp[P - 1]);
      __syncwarp();
      mbar_arrive(ready + s);
    };
    for (; issued < fill; ++issued) {
      // at most kAhead stages in flight while the ring fills: the memory system then
      // returns this CTA's stages in order, so the first one lands early
      if (issued >= kAhead) relay(tr++);
      if (lane == 0) {
        const int sl = sl0 + issued * kSPS;
        issue_stage<WS, P>(maps, stages + (issued % p.S) * L::kStageBytes, full + issued % p.S, sl * kSliceRows,
                           min(kSPS, sl1 - sl), ey, ex, pol);
      }
      __syncwarp();
    }
    for (; tr < nst; ++tr) {
      relay(tr);
      // refill: stage `issued` reuses the slot of stage issued - S, which the consumers
      // release when they are done with it (at most one stage behind this relay)
      while (issued < nst && issued - p.S <= tr - 1) {
        if (lane == 0) {
          const int old = issued - p.S;
          if (!mbar_wait(empty + old % p.S, (old / p.S) & 1) && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
          const int sl = sl0 + issued * kSPS;
          issue_stage<WS, P>(maps, stages + (issued % p.S) * L::kStageBytes, full + issued % p.S, sl * kSliceRows,
                             min(kSPS, sl1 - sl), ey, ex, pol);
        }
        __syncwarp();
        ++issued;
      }
    }
    if (p.Ck > 1) {
      cluster_wait();
      cluster_arrive();
      cluster_wait();
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g4 = lane >> 2, t4 = lane & 3;
  const int gl = warp % GS, kg = warp / GS;  // this warp's strip group and k group
  // ldmatrix.x4 rows: matrix mm = lane / 8 is MMA half (mm & 1) of slice j + (mm >> 1) kKG
  // js: slice step between a warp's slices (1 when it takes whole stages, kKG when the
  // group's warps share every stage); j0: its first slice of a stage
  const bool split = p.split != 0;
  const int js = split ? 1 : kKG, j0 = split ? 0 : kg;
  // ldmatrix.x4 rows: matrix mm = lane / 8 is MMA half (mm & 1) of slice j + (mm >> 1) js
  const int mm = lane >> 3;
  const uint32_t lane_off = static_cast<uint32_t>(L::nib(L::row_of(0, 8 * (mm & 1) + (lane & 7))) +
                                                  (mm >> 1) * js * L::kSliceStride + 16 * gl);

  // AS accumulator sets, one per slice in turn: 2 AS NT independent MMA chains per warp
  // hide the tensor-pipe latency; summed in a fixed order after the loop
  constexpr int AS = 4 / NT;
  float acc[AS][2][NT][4];
#pragma unroll
  for (int a = 0; a < AS; ++a)
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][i][nt][c] = 0.0f;
  uint32_t xw[NT];  // this lane's activation words of the warp's first slice of chunk 0
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) xw[nt] = smem_u32(xs) + (nt * 8 + g4) * kXRow + j0 * 32 + 4 * t4;
  // Activation slice -> shared memory [chunk][n][kXRow]: item t = (batch row, k slice),
  // 32 bytes each (for P = 2 the 16 values go even rows first, then odd rows, the
  // order of the weight fragments); four items' loads in flight per thread. Rows N to
  // 8 NT - 1 of the batch tiles are written as zeros, so the MMA B fragments need no
  // per-lane predicate.
  pdl_wait();  // activations may come from the previous grid; all writes follow it
  {
    constexpr int T = kCW * 32;
    constexpr int kU = 4;
    constexpr int kRows = NT * 8, kRowShift = NT == 1 ? 3 : (NT == 2 ? 4 : 5);
    const int items = (sl1 - sl0) << kRowShift;
    for (int i0 = threadIdx.x; i0 < items; i0 += T * kU) {
      uint4 v[kU][2];
      int so[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int it = i0 + u * T;
        v[u][0] = v[u][1] = make_uint4(0u, 0u, 0u, 0u);
        so[u] = -1;
        if (it < items) {
          const int n = it & (kRows - 1), sl = it >> kRowShift;
          const int k = (sl0 + sl) * kSliceRows;
          const uint4* src = reinterpret_cast<const uint4*>(p.act + static_cast<size_t>(n) * p.K + k);
          if (n < p.N && k < p.K) v[u][0] = __ldg(src);
          if (n < p.N && k + 8 < p.K) v[u][1] = __ldg(src + 1);
          so[u] = (sl >> 3) * p.xcstride + n * kXRow + (sl & 7) * 32;
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (so[u] < 0) continue;
        uint4 a = v[u][0], b = v[u][1];
        if constexpr (P == 2) {
          const uint4 e = make_uint4(prmt(a.x, a.y, 0x5410u), prmt(a.z, a.w, 0x5410u), prmt(b.x, b.y, 0x5410u),
                                     prmt(b.z, b.w, 0x5410u));
          const uint4 o = make_uint4(prmt(a.x, a.y, 0x7632u), prmt(a.z, a.w, 0x7632u), prmt(b.x, b.y, 0x7632u),
                                     prmt(b.z, b.w, 0x7632u));
          a = e;
          b = o;
        }
        *reinterpret_cast<uint4*>(xs + so[u]) = a;
        *reinterpret_cast<uint4*>(xs + so[u] + 16) = b;
      }
    }
  }
  named_bar_sync(1, kCW * 32);

  // per-warp bases: slot 0 of the ring, the warp's first slice; every offset inside a
  // stage below is a compile-time constant, and the slot / parity advance incrementally
  const NibConst kc;
  const uint32_t wbase = smem_u32(stages) + lane_off + j0 * L::kSliceStride;
  const uint32_t scw = smem_u32(scb) + ((j0 * GS + gl) * 4 + t4) * 8;
  // a full stage, slices j0 + i * JS: every ldmatrix of the warp first, then the slices
  auto full_stage = [&](auto jsc, uint32_t sw, uint32_t scs) {
    constexpr int JS = decltype(jsc)::value;
    constexpr int kIt = kSPS / (2 * JS);
    uint32_t w[kIt][4];
#pragma unroll
    for (int it = 0; it < kIt; ++it)
      ldsm_x4_trans(sw + 2 * JS * it * L::kSliceStride, w[it][0], w[it][1], w[it][2], w[it][3]);
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int jr = (2 * it + h) * JS;  // slice offset from the warp's first slice
        const uint2 sc = ld_shared_v2(scs + jr * GS * 32);
        uint32_t xr[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) xr[nt] = xw[nt] + jr * 32;
        consume_slice<NT>(kc, w[it][2 * h], w[it][2 * h + 1], xr, sc, acc[(2 * it + h) % AS]);
      }
    }
  };
  int s = 0;
  uint32_t par = 0;
  for (int st = 0; st < nst; ++st) {
    if (!split || (st & (kKG - 1)) == kg) {
      if (!mbar_wait(ready + s, par) && lane == 0 && p.err) atomicOr(p.err, MB_DEVERR_TIMEOUT);
      const uint32_t sw = wbase + s * L::kStageBytes;
      const uint32_t scs = scw + s * L::kScBytes;
      const int n = min(kSPS, sl1 - (sl0 + st * kSPS));
      if (n == kSPS) {
        if (split)
          full_stage(std::integral_constant<int, 1>(), sw, scs);
        else
          full_stage(std::integral_constant<int, kKG>(), sw, scs);
      } else {
        for (int jr = 0; j0 + jr < n; jr += 2 * js) {
          // lanes 16-31 address slice jr + js; past the stage's last slice they re-read
          // slice jr instead (the rows stay inside the stage; the words are not used)
          const bool hi = j0 + jr + js < n;
          const uint32_t back = (!hi && (lane >> 4)) ? js * L::kSliceStride : 0u;
          uint32_t w0, w1, w2, w3;
          ldsm_x4_trans(sw + jr * L::kSliceStride - back, w0, w1, w2, w3);
          {
            const uint2 sc = ld_shared_v2(scs + jr * GS * 32);
            uint32_t xr[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) xr[nt] = xw[nt] + jr * 32;
            consume_slice<NT>(kc, w0, w1, xr, sc, acc[0]);
          }
          if (hi) {
            const uint2 sc = ld_shared_v2(scs + (jr + js) * GS * 32);
            uint32_t xr[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) xr[nt] = xw[nt] + (jr + js) * 32;
            consume_slice<NT>(kc, w2, w3, xr, sc, acc[AS > 1 ? 1 : 0]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) xw[nt] += p.xcstride;
    if (++s == p.S) {
      s = 0;
      par ^= 1u;
    }
  }

#pragma unroll
  for (int a = 1; a < AS; ++a)
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[0][i][nt][c] += acc[a][i][nt][c];

  // ---- partial tiles -> the owner CTA's receive slots ----
  // owner of strip group g: CTA (g Ck) / GS of the cluster; its groups start at
  // ceil(o GS / Ck). Slot (sender q, k group kg) holds [N][rp] floats.
  const int own = p.owner[gl];
  const int gfo = p.gfirst[own];
  const int col = (gl - gfo) * 32 + 4 * g4;
  const uint32_t slot = smem_u32(recv) + static_cast<uint32_t>((q * kKG + kg) * p.N * p.rp + col) * 4u;
  if (p.Ck > 1) cluster_wait();  // phase 0: every CTA of the cluster runs
  const uint32_t dst = p.Ck > 1 ? mapa_shared(slot, static_cast<uint32_t>(own)) : slot;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int n0 = nt * 8 + 2 * t4;
    const float(&t0)[4] = acc[0][0][nt];
    const float(&t1)[4] = acc[0][1][nt];
    if (n0 < p.N) st_cluster_v4(dst + static_cast<uint32_t>(n0 * p.rp) * 4u, t0[0], t0[2], t1[0], t1[2]);
    if (n0 + 1 < p.N) st_cluster_v4(dst + static_cast<uint32_t>((n0 + 1) * p.rp) * 4u, t0[1], t0[3], t1[1], t1[3]);
  }
  if (p.Ck > 1) {
    cluster_arrive();  // phase 1 (release): this CTA's partials are in their owners' slots
    cluster_wait();
  } else {
    named_bar_sync(1, kCW * 32);
  }

  // ---- owner: add the slots of its columns in (sender, k group) order ----
  const int gf = p.gfirst[q];
  const int c4n = (p.gfirst[q + 1] - gf) * 8;  // 4-column units this CTA owns per batch row (<= 64)
  const int nslot = p.Ck * kKG;
  const int c4 = threadIdx.x & 63;
  for (int n = threadIdx.x >> 6; c4 < c4n && n < p.N; n += kCW * 32 / 64) {
    const float* src = recv + n * p.rp + 4 * c4;
    float4 sum = *reinterpret_cast<const float4*>(src);
    for (int sidx = 1; sidx < nslot; ++sidx) {
      const float4 v = *reinterpret_cast<const float4*>(src + sidx * p.N * p.rp);
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
    }
    if constexpr (XCH) {
      // the same fp16 rounding as the stored output; the epoch was advanced by the
      // previous join of this channel, which completed before pdl_wait above returned
      const int row = p.xrow0 + n;
      const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(p.xstate + row) + 1u;
      const __half2 lo = __floats2half2_rn(sum.x, sum.y), hi = __floats2half2_rn(sum.z, sum.w);
      const uint32_t wlo = *reinterpret_cast<const uint32_t*>(&lo), whi = *reinterpret_cast<const uint32_t*>(&hi);
      const long long e = static_cast<long long>(row) * p.M + c0 + gf * 32 + 4 * c4;  // even word pair
      for (int r = 0; r < p.xworld; ++r) {
        uint2* d = peer_row_slot(p.xbuf[r], static_cast<int>(epoch & 1u), p.xrank, p.xslot) + e / 2;
        st_ll(d, wlo, epoch);
        st_ll(d + 1, whi, epoch);
      }
    } else {
      store_half4(p.out + static_cast<size_t>(n) * p.M + c0 + gf * 32 + 4 * c4, sum.x, sum.y, sum.z, sum.w);
    }
  }
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
  int ws = 0, P = 1, Ck = 1, nt = 1, S = 0, smem = 0, ctas = 0;
  int xcstride = 0, scboff = 0, xoff = 0, recvoff = 0, baroff = 0, rp = 0;
  bool fast = false;
};

static int stage_bytes_of(int ws, int P) {
  if (ws == 256) return Layout<256, 1>::kStageBytes;
  return P == 1 ? Layout<128, 1>::kStageBytes : Layout<128, 2>::kStageBytes;
}

static inline int round_up(int x, int a) { return (x + a - 1) / a * a; }

// The complete launch plan of one (strip width, cluster size) candidate: ring depth and
// shared-memory layout. pl.fast is false if it does not fit.
//  [ring S x stage][scale pairs S x kScBytes][activations: chunks x N x 272 B]
//  [receive slots Ck x kKG x N x rp floats][mbarriers full/empty/ready]
static Plan make_plan(int N, int KS, int P, int ws, int ck) {
  Plan pl;
  pl.nt = N <= 8 ? 1 : (N <= 16 ? 2 : 4);
  pl.P = P;
  pl.ws = ws;
  pl.Ck = ck;
  const int gs = ws / 32, kkg = kCW / gs;
  const int ngmax = (gs + ck - 1) / ck;  // most groups a CTA of the cluster owns
  pl.rp = ngmax * 32 + 4;
  pl.xcstride = round_up(pl.nt * 8 * kXRow, 128);  // batch rows padded to the MMA tiles
  const int KSc = (KS + ck - 1) / ck;        // most k slices a CTA of the cluster gets
  const int need = (KSc + kSPS - 1) / kSPS;  // stages (= activation chunks) of the CTA's slice
  const int xbytes = need * pl.xcstride;
  const int recvbytes = ck * kkg * N * pl.rp * 4;
  const int stage = stage_bytes_of(ws, P) + (ws / 32) * kSPS * 32;  // weights + re-laid scales
  const int fixed = 1024 + xbytes + recvbytes + 3 * kMaxStages * 8;
  const int want = std::min(kMaxStages, need);
  const int S = std::min(want, (227 * 1024 - fixed) / stage);
  // the producer's refill order needs two slots unless the CTA's slice is one stage
  if (S < std::min(2, want) || need < 1) return pl;
  pl.S = S;
  pl.scboff = S * stage_bytes_of(ws, P);
  pl.xoff = round_up(pl.scboff + S * (ws / 32) * kSPS * 32, 128);
  pl.recvoff = round_up(pl.xoff + xbytes, 16);
  pl.baroff = round_up(pl.recvoff + recvbytes, 16);
  pl.smem = 1024 + pl.baroff + 3 * kMaxStages * 8;
  pl.fast = pl.smem <= 227 * 1024;
  return pl;
}

template <int NT, int WS, int P>
static int max_clusters_q(int ck, int smem) {
  auto kern = k_gemm_int4<NT, WS, P, false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ck * 16);
  cfg.blockDim = dim3((kCW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = ck;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  return n;
}

// How many clusters of a plan the GPU holds at once (cudaOccupancyMaxActiveClusters on
// the plan's own kernel). Without a device: the counts measured on B200 for one CTA per
// SM (clusters of 7 and 8 fit only 15 times: a GPC holds two), scaled to the SM count.
static int max_clusters(const Plan& pl, int sms) {
  int n = -1;
#define MB_Q(NT_, WS_, P_) \
  if (pl.nt == NT_ && pl.ws == WS_ && pl.P == P_) n = max_clusters_q<NT_, WS_, P_>(pl.Ck, pl.smem);
  MB_Q(1, 256, 1) MB_Q(1, 128, 1) MB_Q(1, 128, 2) MB_Q(2, 256, 1) MB_Q(2, 128, 1) MB_Q(2, 128, 2)
  MB_Q(4, 256, 1) MB_Q(4, 128, 1) MB_Q(4, 128, 2)
#undef MB_Q
  if (n > 0) return n;
  static const int solo148[kMaxCk + 1] = {0, 148, 74, 45, 33, 26, 22, 15, 15};
  return solo148[pl.Ck] * sms / 148;
}

// Estimated time (ns) of one call under a plan:
//  * a fixed cost (launch hand-off, activation copy, cross-CTA reduction);
//  * the dequant + MMA loop at a rate per SM per cycle that falls with the batch tiles
//    (more MMAs and activation multiplies per weight), ~1.9 GHz;
//  * the weight stream at ~6.5 TB/s as a floor;
//  * a grid larger than what the GPU holds at once runs in more waves.
static double plan_cost(const Plan& pl, int N, int K, int M, int KS, int sms) {
  const int KSc = (KS + pl.Ck - 1) / pl.Ck;
  const double w_cta = static_cast<double>(pl.ws) * KSc * kSliceRows;
  const double rate = pl.nt == 1 ? 56.0 : (pl.nt == 2 ? 45.0 : 32.0);  // weights per cycle per SM
  int waves = 1;
  if (pl.Ck == 1) {
    waves = (pl.ctas + sms - 1) / sms;
  } else if (pl.ctas / pl.Ck > max_clusters(pl, sms)) {
    waves = 2;
  }
  double t = 1500.0 + waves * w_cta / rate / 1.9;
  const double bytes = static_cast<double>(K) * M * kSB / 256 + 2.0 * N * (K + M);
  t = std::max(t, 800.0 + bytes / 6500.0);  // 6.5 TB/s = 6500 bytes per ns
  return t;
}

// Picks the strip width and K split (cluster size) with the lowest estimated time;
// ties go to the wider strip and fewer CTAs per cluster.
static Plan plan_gemm_uncached(int N, int K, int M, int sms) {
  Plan best;
  best.nt = N <= 8 ? 1 : (N <= 16 ? 2 : 4);
  if (K % 8 != 0 || M % 128 != 0) return best;
  const int P = (M % 256 == 0) ? 1 : 2;
  const int KS = (K + kSliceRows - 1) / kSliceRows;
  double best_t = 0.0;
  for (int ws : {256, 128}) {
    if (ws == 256 && P != 1) continue;
    const int strips = M / ws;
    for (int ck = 1; ck <= kMaxCk && ck <= KS; ++ck) {
      const long long ctas = static_cast<long long>(strips) * ck;
      if (ck > 1 && ctas > sms) break;  // a cluster grid must fit one wave
      Plan pl = make_plan(N, KS, P, ws, ck);
      if (!pl.fast) continue;
      pl.ctas = static_cast<int>(ctas);
      const double t = plan_cost(pl, N, K, M, KS, sms);
      if (!best.fast || t < best_t - 1e-6) {
        best = pl;
        best_t = t;
      }
    }
  }
  // Without a K split and in several waves, a CTA takes about the same time per
  // 128-row stage whatever its strip width (measured: a wave of 256-wide strips as
  // long as one of 128-wide strips), so the wider strip halves the waves.
  if (best.fast && best.Ck == 1 && best.ws == 128 && P == 1 && best.ctas > sms) {
    Plan wide = make_plan(N, KS, P, 256, 1);
    if (wide.fast) {
      wide.ctas = M / 256;
      best = wide;
    }
  }
  return best;
}

// Plans are cached per (device, N, K, M): the capacity query is not free and a decode
// loop repeats a handful of shapes.
static Plan plan_gemm(int N, int K, int M, int sms) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    dev = -1;
  }
  const uint64_t key = (static_cast<uint64_t>(static_cast<uint32_t>(dev) & 0xFF) << 56) ^
                       (static_cast<uint64_t>(N) << 48) ^ (static_cast<uint64_t>(static_cast<uint32_t>(K)) << 24) ^
                       static_cast<uint64_t>(static_cast<uint32_t>(M));
  static std::mutex mu;
  static std::unordered_map<uint64_t, Plan> cache;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const Plan pl = plan_gemm_uncached(N, K, M, sms);
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, pl);
  return pl;
}

// Tensor maps of a weight stream: 3-D view [144 bytes][super-blocks per period]
// [periods of P rows], full-stage and 16-row boxes. Encoding costs a few microseconds
// of host time per launch, so maps are cached per (address, K, M, strip, phases): a
// decode loop streams the same weight tensors every step. A map depends only on these
// values, so a cached entry stays valid for any tensor at that address and shape.
template <int WS, int P>
static bool weight_maps(const uint8_t* sb, int K, int M, WMaps* maps) {
  using L = Layout<WS, P>;
  struct Key {
    const uint8_t* sb;
    int K, M;
    bool operator==(const Key& o) const { return sb == o.sb && K == o.K && M == o.M; }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.sb) ^ (static_cast<size_t>(k.K) * 0x9E3779B97F4A7C15ull) ^
             (static_cast<size_t>(k.M) << 1);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, WMaps, Hash> cache;
  const Key key{sb, K, M};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *maps = it->second;
      return true;
    }
  }
  const uint64_t sbp = static_cast<uint64_t>(P) * M / 256;
  const uint64_t dims[3] = {kSB, sbp, static_cast<uint64_t>(K / P)};
  const uint64_t strides[2] = {kSB, sbp * kSB};
  bool ok;
  if (WS == 256) {
    const uint32_t bf[3] = {kSB, 1, kStageRows}, bs[3] = {kSB, 1, kSliceRows};
    ok = encode_tmap_3d_u8(&maps->full_a, sb, dims, strides, bf) &&
         encode_tmap_3d_u8(&maps->slice_a, sb, dims, strides, bs);
    maps->full_b = maps->full_a;
    maps->slice_b = maps->slice_a;
  } else {
    const uint32_t sf[3] = {16, 1, kStageRows / P}, ss[3] = {16, 1, kSliceRows / P};
    const uint32_t nf[3] = {L::kNibRow, 1, kStageRows / P}, ns[3] = {L::kNibRow, 1, kSliceRows / P};
    ok = encode_tmap_3d_u8(&maps->full_a, sb, dims, strides, sf) &&
         encode_tmap_3d_u8(&maps->slice_a, sb, dims, strides, ss) &&
         encode_tmap_3d_u8(&maps->full_b, sb, dims, strides, nf) &&
         encode_tmap_3d_u8(&maps->slice_b, sb, dims, strides, ns);
  }
  if (!ok) return false;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() >= 4096) cache.clear();
  cache.emplace(key, *maps);
  return true;
}

// x: the exchange of an XCH launch (its fields of GemmParams), else null.
template <int NT, int WS, int P, bool XCH>
static int launch_fast(const Plan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
                       uint32_t* err, cudaStream_t st, const GemmParams* x) {
  auto kern = k_gemm_int4<NT, WS, P, XCH>;
  static bool attr_set[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MB_ERR_LAUNCH;
  if (!attr_set[dev]) {
    // full shared-memory carveout: the ring, activations and receive slots share it
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return MB_ERR_LAUNCH;
    attr_set[dev] = true;
  }
  WMaps maps;
  if (!weight_maps<WS, P>(sb, K, M, &maps)) return MB_ERR_LAUNCH;
  GemmParams prm;
  if (XCH) {
    for (int r = 0; r < kPeerMaxRanks; ++r) prm.xbuf[r] = x->xbuf[r];
    prm.xstate = x->xstate;
    prm.xslot = x->xslot;
    prm.xworld = x->xworld;
    prm.xrank = x->xrank;
    prm.xrow0 = x->xrow0;
  } else {
    for (int r = 0; r < kPeerMaxRanks; ++r) prm.xbuf[r] = nullptr;
    prm.xstate = nullptr;
    prm.xslot = 0;
    prm.xworld = prm.xrank = prm.xrow0 = 0;
  }
  prm.out = out;
  prm.act = act;
  prm.err = err;
  prm.N = N;
  prm.K = K;
  prm.M = M;
  prm.KS = (K + kSliceRows - 1) / kSliceRows;
  prm.Ck = pl.Ck;
  prm.S = pl.S;
  prm.xcstride = pl.xcstride;
  prm.scboff = pl.scboff;
  prm.xoff = pl.xoff;
  prm.recvoff = pl.recvoff;
  prm.baroff = pl.baroff;
  prm.rp = pl.rp;
  for (int q = 0; q <= kMaxCk; ++q) {
    const int qq = std::min(q, pl.Ck);
    prm.sl_first[q] = static_cast<int>((static_cast<long long>(qq) * prm.KS) / pl.Ck);
    prm.gfirst[q] = (qq * (WS / 32) + pl.Ck - 1) / pl.Ck;
  }
  for (int g = 0; g < 8; ++g) prm.owner[g] = (g * pl.Ck) / (WS / 32);
  // whole stages per warp for one batch tile when every warp of a group gets at least
  // two of them (measured: faster at N <= 8, slower with more batch tiles)
  const int kkg = kCW / (WS / 32);
  const int need = ((prm.KS + pl.Ck - 1) / pl.Ck + kSPS - 1) / kSPS;
  prm.split = (NT == 1 && need >= 2 * kkg) ? 1 : 0;

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

template <int NT, bool XCH = false>
static int dispatch_fast(const Plan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
                         uint32_t* err, cudaStream_t st, const GemmParams* x = nullptr) {
  if (pl.ws == 256) return launch_fast<NT, 256, 1, XCH>(pl, act, sb, out, N, K, M, err, st, x);
  if (pl.ws == 128)
    return pl.P == 1 ? launch_fast<NT, 128, 1, XCH>(pl, act, sb, out, N, K, M, err, st, x)
                     : launch_fast<NT, 128, 2, XCH>(pl, act, sb, out, N, K, M, err, st, x);
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

// One launch over up to 32 batch rows: the cluster kernel, else the generic one.
static int gemm_rows(const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M, uint32_t* err,
                     cudaStream_t st) {
  if (aligned(act, 16) && aligned(sb, 16) && aligned(out, 4)) {
    const Plan pl = plan_gemm(N, K, M, sm_count());
    if (pl.fast) {
      if (pl.nt == 1) return dispatch_fast<1>(pl, act, sb, out, N, K, M, err, st);
      if (pl.nt == 2) return dispatch_fast<2>(pl, act, sb, out, N, K, M, err, st);
      return dispatch_fast<4>(pl, act, sb, out, N, K, M, err, st);
    }
  }
  return launch_generic(act, sb, out, N, K, M, st);
}

static int gemm_all(const uint16_t* act, const uint8_t* sb, uint16_t* out, int32_t N, int32_t K, int32_t M,
                    uint32_t* dev_err, void* stream) {
  if (N < 1 || K < 1 || M < 1 || (static_cast<int64_t>(K) * M) % 256 != 0) return MB_ERR_ARGS;
  if (!act || !sb || !out) return MB_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Rows per launch: 32, or 16 where a block of more than 16 rows does not fit the fast
  // plan but 16 rows do (a wide matrix without a K split and a long K: the activations
  // of the whole K for 32 rows leave no room for the ring), since two fast launches
  // beat one of the generic kernel by far.
  int rb = 32;
  if (N > 16 && !plan_gemm(std::min(N, 32), K, M, sm_count()).fast && plan_gemm(16, K, M, sm_count()).fast) rb = 16;
  for (int r0 = 0; r0 < N; r0 += rb) {
    const int nb = std::min(rb, N - r0);
    const int rc = gemm_rows(act + static_cast<size_t>(r0) * K, sb, out + static_cast<size_t>(r0) * M, nb, K, M,
                             dev_err, st);
    if (rc != MB_OK) return rc;
  }
  return MB_OK;
}

}  // namespace mb

using namespace mb;

extern "C" {

int32_t mb_int4_gemm(const uint16_t* act, const uint8_t* sb, uint16_t* out, int32_t N, int32_t K, int32_t M,
                     uint32_t* dev_err, void* stream) {
  return gemm_all(act, sb, out, N, K, M, dev_err, stream);
}

int32_t mb_int4_gemm_peer(const uint16_t* act, const uint8_t* sb, int32_t N, int32_t K, int32_t M,
                          void* const* bufs, int32_t world, int32_t rank, int64_t slot_elems, const uint32_t* state,
                          uint32_t* dev_err, void* stream) {
  if (!act || !sb || !bufs || !state) return MB_ERR_NULL;
  if (N < 1 || N > kPeerMaxRows || K < 1 || M < 8 || M % 8 != 0 || (static_cast<int64_t>(K) * M) % 256 != 0 ||
      world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world || slot_elems % 8 != 0 ||
      static_cast<int64_t>(N) * M > slot_elems)
    return MB_ERR_ARGS;
  GemmParams x;
  for (int r = 0; r < kPeerMaxRanks; ++r) {
    x.xbuf[r] = r < world ? static_cast<uint8_t*>(bufs[r]) : nullptr;
    if (r < world && (!bufs[r] || !aligned(bufs[r], 256))) return MB_ERR_ARGS;
  }
  if (!aligned(act, 16) || !aligned(sb, 16)) return MB_ERR_UNSUPPORTED;  // the fast plan only
  x.xstate = state;
  x.xslot = slot_elems;
  x.xworld = world;
  x.xrank = rank;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int r0 = 0; r0 < N; r0 += 32)  // every block on the fast plan before anything is launched
    if (!plan_gemm(std::min(32, N - r0), K, M, sm_count()).fast) return MB_ERR_UNSUPPORTED;
  for (int r0 = 0; r0 < N; r0 += 32) {
    const int nb = std::min(32, N - r0);
    const Plan pl = plan_gemm(nb, K, M, sm_count());
    x.xrow0 = r0;
    const uint16_t* a = act + static_cast<size_t>(r0) * K;
    const int rc = pl.nt == 1   ? dispatch_fast<1, true>(pl, a, sb, nullptr, nb, K, M, dev_err, st, &x)
                   : pl.nt == 2 ? dispatch_fast<2, true>(pl, a, sb, nullptr, nb, K, M, dev_err, st, &x)
                                : dispatch_fast<4, true>(pl, a, sb, nullptr, nb, K, M, dev_err, st, &x);
    if (rc != MB_OK) return rc;
  }
  return MB_OK;
}

int32_t mb_int4_gemm_host(const uint16_t* act_host, const uint8_t* sb, uint16_t* out_host, int32_t N, int32_t K,
                          int32_t M, uint16_t* act_dev, uint16_t* out_dev, uint32_t* dev_err, void* stream) {
  if (!act_host || !sb || !out_host || !act_dev || !out_dev) return MB_ERR_NULL;
  if (N < 1 || K < 1 || M < 1 || (static_cast<int64_t>(K) * M) % 256 != 0) return MB_ERR_ARGS;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t in_bytes = static_cast<size_t>(N) * K * 2, out_bytes = static_cast<size_t>(N) * M * 2;
  if (cudaMemcpyAsync(act_dev, act_host, in_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  const int32_t rc = gemm_all(act_dev, sb, out_dev, N, K, M, dev_err, stream);
  if (rc != MB_OK) return rc;
  if (cudaMemcpyAsync(out_host, out_dev, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return MB_OK;
}

// Host-buffer calls that overlap one another: per (device, caller stream) a pipe of two
// library-owned copy streams and MB_HOST_SLOTS staging slots. Call i copies its input
// into slot i % MB_HOST_SLOTS on the input stream, the caller's stream waits for that
// copy and runs the GEMM, and the output stream waits for the GEMM and copies the
// result out; each slot's next input copy waits for its previous output copy. So the
// input copy of the next call and the output copy of the previous one run beside
// the current GEMM (separate copy engines), and no slot is overwritten while in use.
constexpr int kHostSlots = MB_HOST_SLOTS;
struct HostPipe {
  cudaStream_t s_in = nullptr, s_out = nullptr;
  cudaEvent_t ev_in[kHostSlots] = {}, ev_k[kHostSlots] = {}, ev_out[kHostSlots] = {};
  uint32_t next = 0;
};

static HostPipe* host_pipe(cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  const uint64_t key = (static_cast<uint64_t>(dev & 0xFF) << 56) ^ static_cast<uint64_t>(reinterpret_cast<uintptr_t>(st));
  static std::mutex mu;
  static std::unordered_map<uint64_t, HostPipe*> pipes;
  std::lock_guard<std::mutex> lk(mu);
  auto it = pipes.find(key);
  if (it != pipes.end()) return it->second;
  HostPipe* p = new HostPipe();
  bool ok = cudaStreamCreateWithFlags(&p->s_in, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&p->s_out, cudaStreamNonBlocking) == cudaSuccess;
  for (int i = 0; ok && i < kHostSlots; ++i)
    ok = cudaEventCreateWithFlags(&p->ev_in[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&p->ev_k[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&p->ev_out[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    (void)cudaGetLastError();
    return nullptr;  // leaked on failure: a process that cannot create streams has bigger problems
  }
  pipes.emplace(key, p);
  return p;
}

static inline size_t host_slot_in(int32_t N, int32_t K) { return (static_cast<size_t>(N) * K * 2 + 255) / 256 * 256; }
static inline size_t host_slot_bytes(int32_t N, int32_t K, int32_t M) {
  return host_slot_in(N, K) + (static_cast<size_t>(N) * M * 2 + 255) / 256 * 256;
}

size_t mb_int4_gemm_host_staging_bytes(int32_t N, int32_t K, int32_t M) {
  if (N < 1 || K < 1 || M < 1) return 0;
  return static_cast<size_t>(kHostSlots) * host_slot_bytes(N, K, M);
}

int32_t mb_int4_gemm_host_overlap(const uint16_t* act_host, const uint8_t* sb, uint16_t* out_host, int32_t N,
                                  int32_t K, int32_t M, void* staging, size_t staging_bytes, uint32_t* dev_err,
                                  void* stream) {
  if (!act_host || !sb || !out_host || !staging) return MB_ERR_NULL;
  if (N < 1 || K < 1 || M < 1 || (static_cast<int64_t>(K) * M) % 256 != 0) return MB_ERR_ARGS;
  if (!aligned(staging, 256)) return MB_ERR_ALIGN;
  const size_t slot = (staging_bytes / kHostSlots) / 256 * 256;  // slots of a fixed size whatever the shape
  if (host_slot_bytes(N, K, M) > slot) return MB_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  HostPipe* p = host_pipe(st);
  if (!p) return MB_ERR_LAUNCH;
  const int s = static_cast<int>(p->next++ % kHostSlots);
  uint8_t* base = static_cast<uint8_t*>(staging) + static_cast<size_t>(s) * slot;
  uint16_t* in = reinterpret_cast<uint16_t*>(base);
  uint16_t* out = reinterpret_cast<uint16_t*>(base + host_slot_in(N, K));
  const size_t in_bytes = static_cast<size_t>(N) * K * 2, out_bytes = static_cast<size_t>(N) * M * 2;
  if (cudaStreamWaitEvent(p->s_in, p->ev_out[s], 0) != cudaSuccess ||
      cudaMemcpyAsync(in, act_host, in_bytes, cudaMemcpyHostToDevice, p->s_in) != cudaSuccess ||
      cudaEventRecord(p->ev_in[s], p->s_in) != cudaSuccess || cudaStreamWaitEvent(st, p->ev_in[s], 0) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  const int32_t rc = gemm_all(in, sb, out, N, K, M, dev_err, stream);
  if (rc != MB_OK) return rc;
  if (cudaEventRecord(p->ev_k[s], st) != cudaSuccess || cudaStreamWaitEvent(p->s_out, p->ev_k[s], 0) != cudaSuccess ||
      cudaMemcpyAsync(out_host, out, out_bytes, cudaMemcpyDeviceToHost, p->s_out) != cudaSuccess ||
      cudaEventRecord(p->ev_out[s], p->s_out) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return MB_OK;
}

int32_t mb_int4_gemm_host_wait(void* stream) {
  HostPipe* p = host_pipe(static_cast<cudaStream_t>(stream));
  if (!p) return MB_ERR_LAUNCH;
  if (cudaStreamSynchronize(p->s_in) != cudaSuccess || cudaStreamSynchronize(p->s_out) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return MB_OK;
}

int32_t mb_int4_gemm_plan(int32_t N, int32_t K, int32_t M, int32_t* info) {
  if (!info) return MB_ERR_NULL;
  if (N < 1 || K < 1 || M < 1) return MB_ERR_ARGS;
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
