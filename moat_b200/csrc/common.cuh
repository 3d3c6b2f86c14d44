// Shared device helpers for the moat_b200 kernels (sm_100a only).
//
// Inline PTX wrappers for mbarriers, tensor-map (TMA) bulk loads, programmatic
// dependent launch, warp-level mma and the nibble -> fp16 expansion used by every
// INT4 kernel. Status codes follow the reference C ABI's convention of negative
// integers for argument errors (antigravity_c_api.h:129-130: -1 null / not loaded,
// -2 invalid arguments) and extend it.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/moat_b200.h"

namespace mb {

// ---------------------------------------------------------------------------
// Host-side helpers
// ---------------------------------------------------------------------------
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MB_OK : MB_ERR_LAUNCH;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Encode a 3-D tiled uint8 tensor map (dims inner -> outer, strides of dims 1 and 2 in
// bytes). Returns false if the driver rejects the parameters.
bool encode_tmap_3d_u8(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides[2],
                       const uint32_t box[3]);

// Number of SMs of the current device (cached per device).
int sm_count();

// Encode a 2-D tiled tensor map through the driver entry point (no -lcuda link).
// Returns false if the driver rejects the parameters.
bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                    uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swizzle);

// ---------------------------------------------------------------------------
// Device-side helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Every wait in these kernels is bounded: after kWaitBudget cycles it gives up and
// reports false, the caller records MB_DEVERR_TIMEOUT and carries on so the grid
// always terminates.
constexpr long long kWaitBudget = 4000000000LL;  // ~2 s at 2 GHz

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitBudget) return false;
  }
  return true;
}

// L2 cache policies for TMA loads: streamed weights are read once (evict first),
// activations are re-read by every CTA (evict last).
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

// 2-D tiled TMA load (global -> this CTA's shared memory), completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// Programmatic dependent launch: let the next grid on the stream start its
// prologue early / wait until the previous grid has finished and flushed memory.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Host: launch `kern` with programmatic dependent launch allowed, so it may start while
// its predecessor on the stream finishes; the kernel must call pdl_wait() before it
// touches anything the predecessor writes.
template <typename Kern, typename... Args>
inline int launch_with_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, args...) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  return MB_OK;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <uint32_t LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Expand the low nibbles of bytes 0 and 2 of `p` into half2 (n0 - 8, n2 - 8) and the
// high nibbles into half2 (h0 - 8, h2 - 8). Exact: 1024 + n (and 1024 + 16 n) are
// fp16 integers, the magic exponent is removed by an exact subtract / fma.
__device__ __forceinline__ void nibbles_to_half2(uint32_t p, uint32_t& lo, uint32_t& hi) {
  const uint32_t l = lop3<0xEA>(p, 0x000F000Fu, 0x64006400u);  // (p & mask) | magic
  const uint32_t h = lop3<0xEA>(p, 0x00F000F0u, 0x64006400u);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(l), "r"(0x64086408u));                  // - 1032
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(hi) : "r"(h), "r"(0x2C002C00u), "r"(0xD480D480u));  // /16 - 72
}

// D[16x8] += A[16x16] * B[16x8], fp16 in, fp32 accumulate. A pure register
// operation: not volatile, so the compiler may interleave it with the next slice's
// loads across a barrier wait.
__device__ __forceinline__ void mma_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__device__ __forceinline__ void red_add_v2(float* addr, float a, float b) {
  asm volatile("red.relaxed.gpu.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b) : "memory");
}


// ---------------------------------------------------------------------------
// Greedy-choice keys (numpy.argmax rules over fp16: NaN largest, -0 == +0, ties to
// the first column): key = code << 32 | (0xFFFFFFFF - column), code an order-preserving
// 16-bit image of the value, so the largest key names the argmax.
__device__ __forceinline__ uint32_t argmax_code16(uint16_t h) {
  if ((h & 0x7C00u) == 0x7C00u && (h & 0x03FFu)) return 0xFFFFu;
  if (h == 0x8000u) h = 0;
  return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}

__device__ __forceinline__ unsigned long long argmax_key16(uint16_t h, int col) {
  return (static_cast<unsigned long long>(argmax_code16(h)) << 32) | (0xFFFFFFFFull - static_cast<uint32_t>(col));
}

// This thread's best key over row[0, V) (global columns col0 + c), thread `tid` of `nt`:
// 16-byte loads issued four at a time when the row is 16-byte aligned, scalar otherwise.
__device__ __forceinline__ unsigned long long thread_best_key(const uint16_t* __restrict__ row, int V, int col0,
                                                              int tid, int nt) {
  unsigned long long best = 0;
  int c_tail = 0;
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const int nv = V >> 3;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    for (int i0 = tid; i0 < nv; i0 += 4 * nt) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * nt;
        v[u] = i < nv ? __ldg(rv + i) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * nt;
        if (i < nv) {
          const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const unsigned long long k0 = argmax_key16(static_cast<uint16_t>(w[j] & 0xFFFFu), col0 + 8 * i + 2 * j);
            const unsigned long long k1 = argmax_key16(static_cast<uint16_t>(w[j] >> 16), col0 + 8 * i + 2 * j + 1);
            best = k0 > best ? k0 : best;
            best = k1 > best ? k1 : best;
          }
        }
      }
    }
    c_tail = nv << 3;
  }
  for (int c = c_tail + tid; c < V; c += nt) {
    const unsigned long long k = argmax_key16(row[c], col0 + c);
    best = k > best ? k : best;
  }
  return best;
}

// Thread-block cluster helpers (distributed shared memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Full cluster barrier: every thread of every CTA in the cluster arrives (release)
// and waits (acquire), so shared-memory writes before it are visible cluster-wide.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split form of the cluster barrier: every thread of the cluster arrives once and
// waits once per phase (warp-convergent).
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Arrival that orders nothing: for a phase whose only meaning is "this thread got here"
// (a release would first wait for the thread's outstanding global stores).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the async proxy
// (bulk copies issued after a following barrier).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from this CTA's
// shared memory into another CTA of the cluster; `dst` and `remote_bar` are
// shared::cluster addresses (mapa), completion is signalled on the remote mbarrier.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, const void* src, uint32_t bytes,
                                                  uint32_t remote_bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "r"(smem_u32(src)), "r"(bytes), "r"(remote_bar)
      : "memory");
}

// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_cluster_v2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}

// 3-D tiled TMA load (global -> this CTA's shared memory), completion on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

}  // namespace mb

