// Decode attention on a fixed device scratch: an entry point that allocates nothing.
//
// mb_decode_attn asks its caller for a workspace. Some callers cannot hand one over:
//   - a host that binds the C ABI from a language with no device allocator of its
//     own (a cgo or JNI binding that holds only the model's buffers) and keeps no
//     device state between calls;
//   - a serving process whose caching allocator already holds the free HBM, so that a
//     raw device allocation fails, and whose decode loop must not free memory either,
//     because a device free waits for all work on the device to finish.
// mb_decode_attn_noalloc runs the same three kernels (identical results) on a scratch
// array that is part of this module, reserved when the CUDA runtime loads the module
// on a device; the call itself allocates and frees nothing.
//
// Rules of use:
//   - Limit: MB_ATTN_NOALLOC_SCRATCH_BYTES (16 MiB) per device. A shape whose
//     mb_decode_attn_workspace_size() is larger is rejected with MB_ERR_WORKSPACE and
//     nothing is launched (16 traces x 16 heads x 4096 positions x d = 128 needs
//     5,254,400 bytes, about 5.3 MB).
//   - Nothing in the scratch has to start at zero: pass 1 rewrites the per-row
//     arrival counters before pass 3 counts on them, and every other scratch byte is
//     written before it is read.
//   - One scratch per device, shared by every call on that device: two calls that
//     may run at the same time (unordered streams, or several host threads) race on it
//     and can return wrong outputs. Order them (one stream, or events between streams).
//   - The first call on a device resolves the scratch address there
//     (cudaGetSymbolAddress, with that device current) and caches it; make that first
//     call before any stream capture begins on that device.
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace mb {

int32_t decode_attn_enqueue(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int T, int H,
                            int L, int d, float scale, const uint16_t* table, int size, float range_max,
                            void* scratch, cudaStream_t st, int64_t kv_stride, const int32_t* lens,
                            int len_add);

constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(16) << 20;
static_assert(kNoAllocScratchBytes == MB_ATTN_NOALLOC_SCRATCH_BYTES, "header and module disagree on the limit");

static __device__ __align__(256) uint8_t g_attn_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
static std::atomic<void*> g_noalloc_base[kNoAllocMaxDevices];
static std::mutex g_noalloc_mu;

// Address of this device's scratch, resolved once per device (device already current).
static int32_t noalloc_scratch(int dev, void** base) {
  void* p = g_noalloc_base[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    p = g_noalloc_base[dev].load(std::memory_order_relaxed);
    if (!p) {
      const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        (void)cudaGetLastError();
        return MB_ERR_LAUNCH;
      }
      g_noalloc_base[dev].store(p, std::memory_order_release);
    }
  }
  *base = p;
  return MB_OK;
}

}  // namespace mb

using namespace mb;

extern "C" int32_t mb_decode_attn_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                                          int32_t T, int32_t H, int32_t L, int32_t d, float scale,
                                          const uint16_t* table, int32_t size, float range_max, void* stream) {
  if (!q || !k || !v || !out || !table) return MB_ERR_NULL;
  if (T < 1 || H < 1 || L < 1 || d < 8 || d > 256 || d % 8 != 0 || (d & (d - 1)) != 0 || size < 2 ||
      !(range_max > 0.0f))
    return MB_ERR_ARGS;
  if (static_cast<int64_t>(T) * H > 65535) return MB_ERR_UNSUPPORTED;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16)) return MB_ERR_ALIGN;
  if (mb_decode_attn_workspace_size(T, H, L, d) > kNoAllocScratchBytes) return MB_ERR_WORKSPACE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return MB_ERR_LAUNCH;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) return MB_ERR_UNSUPPORTED;
  void* base = nullptr;
  const int32_t rc = noalloc_scratch(dev, &base);
  if (rc != MB_OK) return rc;
  return decode_attn_enqueue(q, k, v, out, T, H, L, d, scale, table, size, range_max, base,
                             static_cast<cudaStream_t>(stream), 0, nullptr, 0);
}
