// xp_decode_step_noalloc: the decode step for callers that cannot allocate
// device memory.
//
// Some callers of this library cannot call cudaMalloc (or ask torch for a
// buffer) when they page a layer: a serving engine that has already handed all
// free device memory to its own allocator (KV cache and activations are
// reserved up front, so a late allocation fails or fragments the pool), or a
// host program in another language that drives the library through the C ABI
// alone and has no device allocator of its own.  This entry point does the same
// work as xp_decode_step followed (for compressed rows) by xp_decode_rows, but
// takes its scratch memory -- the step's flag block and the staging rows of
// the compressed records -- from a fixed array compiled into the library.
//
// The array is XP_NOALLOC_SCRATCH_BYTES (32 MiB) of device memory on every GPU
// that loads the library, held until the process exits.  The flags occupy its
// first 256 bytes; the staging of K compressed rows takes K x (P0 + P1) x 4
// bytes after them, so K x (P0 + P1) x 4 + 256 must not exceed the array
// (8 Qwen-sized rows at pitch 0.89 need 22.4 MB); larger requests are refused
// with XP_ERANGE before anything is launched.
//
// Host code cannot use the array's name as an address: the first call on each
// device looks the address up with cudaGetSymbolAddress, with that device
// current (this may load the library's device code, so that first call should
// come before any stream capture), and queues a clear of the flag block on the
// call's stream, ahead of the kernels the call launches there.  Later calls
// reuse the address, which stays valid for the life of the device's primary
// context: do not call this entry point again after cudaDeviceReset.  Every
// call on a device shares the one array and finds the previous call's contents
// in it: the step kernel leaves the flags at zero (except its give-up counter,
// word 3, which keeps counting across calls), and the staging rows are fully
// rewritten by each call.  Two calls whose work overlaps on the GPU (different
// streams, no ordering between them) race on the array.
//
// A wait of the step that gives up leaves stale staging rows, which the decode
// then expands into slots the tables mark as filled.  The caller learns of it
// through errors_out: when a wait gives up, the kernel stores the running
// give-up count there (device memory, or mapped pinned host memory that the
// host can poll without synchronising).
#include <cuda_runtime.h>

#include <mutex>

#include "xpager.h"

namespace {

constexpr size_t kFlagsBytes = 256;
constexpr int kMaxDevices = 128;
// Staging words that fit after the flag block.
constexpr int64_t kRoomWords = (static_cast<int64_t>(XP_NOALLOC_SCRATCH_BYTES) - 256) / 4;
constexpr int64_t kMaxRows = 2048;  // the step kernel's list limit

static __device__ __align__(256) unsigned char g_scratch[XP_NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
unsigned char *g_addr[kMaxDevices];

// The device address of g_scratch on the current device.  On the first use on
// a device the address is looked up and a clear of the flag block is queued on
// `stream`.
int scratch_address(unsigned char **out, cudaStream_t stream) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return static_cast<int>(err);
  if (dev < 0 || dev >= kMaxDevices) return XP_ERANGE;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void *p = nullptr;
    err = cudaGetSymbolAddress(&p, g_scratch);
    if (err != cudaSuccess) return static_cast<int>(err);
    err = cudaMemsetAsync(p, 0, kFlagsBytes, stream);
    if (err != cudaSuccess) return static_cast<int>(err);
    g_addr[dev] = static_cast<unsigned char *>(p);
  }
  *out = g_addr[dev];
  return XP_OK;
}

}  // namespace

extern "C" int xp_decode_step_noalloc(
    const void *topk_ids, int ids_bytes, int64_t K, int64_t E,
    int64_t *a_slot_of, int64_t *a_expert_in, int64_t *a_last_used, int64_t *a_counters,
    int64_t a_slots, int32_t *expert_map, int64_t *a_slot, int64_t *a_todo,
    int64_t *b_slot_of, int64_t *b_expert_in, int64_t *b_last_used, int64_t *b_counters,
    int64_t b_slots, int64_t *b_slot, int64_t *b_todo,
    const int64_t *no_cache, int64_t base,
    const void *src0, void *dst0, int64_t W0, int64_t P0,
    const void *src1, void *dst1, int64_t W1, int64_t P1,
    const void *scale0, void *sdst0, int64_t SW0, const void *scale1, void *sdst1, int64_t SW1,
    int compress, const uint8_t *lut, int64_t chunk, int ctas, int64_t layer, int64_t *seq,
    int64_t *req, const int64_t *done, int64_t block, int64_t ring, int64_t retry_ns,
    int64_t giveup, uint32_t *errors_out, void *stream) {
  if (K < 0 || P0 < 0 || P1 < 0 || W0 < 0 || W1 < 0) return XP_EINVAL;
  // Staging rows are P words each; keep every row 16-byte aligned.
  if (compress && ((P0 * 4) % 16 || (P1 * 4) % 16)) return XP_EINVAL;
  // Bound each factor before multiplying, so K x (P0 + P1) x 4 cannot wrap.
  if (K > kMaxRows || (compress && (P0 > kRoomWords || P1 > kRoomWords))) return XP_ERANGE;
  const int64_t stage0 = compress ? K * P0 * 4 : 0, stage1 = compress ? K * P1 * 4 : 0;
  if (stage0 + stage1 + static_cast<int64_t>(kFlagsBytes) >
      static_cast<int64_t>(XP_NOALLOC_SCRATCH_BYTES))
    return XP_ERANGE;
  unsigned char *scratch = nullptr;
  int rc = scratch_address(&scratch, static_cast<cudaStream_t>(stream));
  if (rc != XP_OK) return rc;
  unsigned char *stg0 = compress ? scratch + kFlagsBytes : nullptr;
  unsigned char *stg1 = compress ? scratch + kFlagsBytes + stage0 : nullptr;
  rc = xp_decode_step(topk_ids, ids_bytes, K, E, a_slot_of, a_expert_in, a_last_used, a_counters,
                      a_slots, expert_map, nullptr, a_slot, a_todo, b_slot_of, b_expert_in,
                      b_last_used,
                      b_counters, b_slots, b_slot, b_todo, no_cache, base, src0, dst0, stg0, W0,
                      P0, src1, dst1, stg1, W1, P1, scale0, sdst0, SW0, scale1, sdst1, SW1,
                      compress, compress ? chunk : 0, ctas, layer, seq, req, done, block, ring,
                      retry_ns, giveup, reinterpret_cast<uint32_t *>(scratch), errors_out,
                      stream);
  if (rc != XP_OK || !compress || K == 0) return rc;
  return xp_decode_rows(a_todo, K, a_slot, no_cache, lut, stg0, P0 * 4, dst0, W0 * 4, stg1,
                        P1 * 4, dst1, W1 * 4, nullptr, chunk, stream);
}
