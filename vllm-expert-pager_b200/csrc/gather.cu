// Gather of missed expert rows into VRAM slots, and the GPU side of the SSD
// request ring: the C-ABI entry points xp_gather_rows, xp_fetch_publish,
// xp_fetch_wait, xp_fetch.
//
// Semantics follow monochromegane/vllm-expert-pager src/vllm_expert_pager/gather.py.
// The copy is done by the SMs, not a copy engine, so that the rows to move are
// read from device-resident index arrays and the launch replays from a CUDA
// graph (gather.py:15-17).  Device code: gather_dev.cuh.
#include "gather_dev.cuh"

namespace xp {
namespace {

using namespace gdev;

constexpr int kDefaultCtas = 16;

struct GatherArgs {
  CopyJob job;
  int copy_ctas;
  int fetch;  // the last CTA runs the fetch
  Fetch f;
};

__global__ void fetch_kernel(const __grid_constant__ Fetch f, int publish, int wait) {
  if (publish) fetch_publish(f);
  if (publish && wait) __syncthreads();
  if (wait) fetch_wait(f);
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) gather_kernel(const __grid_constant__ GatherArgs a) {
  if (a.fetch && blockIdx.x == gridDim.x - 1) {
    // gather.py:170-185: this CTA asks the host for the SSD reads and waits
    // while the others copy the experts that are in RAM.
    fetch_publish(a.f);
    __syncthreads();
    fetch_wait(a.f);
    return;
  }
  __shared__ CopySmem sm;
  copy_rows<VEC>(a.job, blockIdx.x, a.copy_ctas, sm);
}

bool ring_ok(const int64_t *seq, const int64_t *req, const int64_t *done, int64_t block,
             int64_t ring) {
  return seq && req && done && block >= 1 && ring >= 1;
}

}  // namespace

// Fills the two names of a copy job; returns false on a bad argument.  `vec`
// is cleared when a row or pointer is not 16-byte aligned.
bool fill_names(CopyJob &job, const void *const srcs[2], const void *const caches[2],
                void *const dsts[2], void *const stgs[2], const int64_t Ws[2], const int64_t Ps[2],
                const void *const scales[2], void *const sdsts[2], const int64_t SWs[2],
                int compress, bool &vec) {
  if (!compress && (Ps[0] != Ws[0] || Ps[1] != Ws[1])) return false;
  vec = true;
  for (int i = 0; i < 2; ++i) {
    if (Ws[i] < 0 || Ps[i] < 0 || SWs[i] < 0 || !dsts[i] || !scales[i] || !sdsts[i]) return false;
    if (compress && !stgs[i]) return false;
    Name &n = job.n[i];
    n.src = static_cast<const int32_t *>(srcs[i]);
    n.cache = static_cast<const int32_t *>(caches[i]);
    n.dst = static_cast<int32_t *>(dsts[i]);
    n.stg = static_cast<int32_t *>(stgs[i]);
    n.W = Ws[i];
    n.P = Ps[i];
    const int64_t m = Ws[i] > Ps[i] ? Ws[i] : Ps[i];
    n.C = (m + kPieceWords - 1) / kPieceWords;
    n.scale = static_cast<const int32_t *>(scales[i]);
    n.sdst = static_cast<int32_t *>(sdsts[i]);
    n.SW = SWs[i];
    vec = vec && (Ws[i] % 4 == 0) && (Ps[i] % 4 == 0) && aligned(srcs[i], 16) &&
          aligned(caches[i], 16) && aligned(dsts[i], 16) && (!compress || aligned(stgs[i], 16));
  }
  job.compress = compress;
  return true;
}

}  // namespace xp

using namespace xp;
using namespace xp::gdev;

extern "C" int xp_gather_rows(const int64_t *todo, int64_t K, const int64_t *dst_row,
                              const int64_t *cache_row, const int64_t *src_row, int64_t base,
                              const void *src0, const void *cache0, void *dst0, void *stg0,
                              int64_t W0, int64_t P0, const void *src1, const void *cache1,
                              void *dst1, void *stg1, int64_t W1, int64_t P1, const void *scale0,
                              void *sdst0, int64_t SW0, const void *scale1, void *sdst1,
                              int64_t SW1, const int64_t *skip, int compress, int64_t chunk,
                              int ctas,
                              int64_t layer, int64_t *seq, int64_t *req, const int64_t *done,
                              int64_t block, int64_t ring, int64_t retry_ns, int64_t giveup,
                              void *stream) {
  if (K < 0 || K > kMaxK || (K > 0 && (!todo || !dst_row || !cache_row || !src_row)))
    return XP_EINVAL;
  GatherArgs a{};
  a.job.todo = todo;
  a.job.K = K;
  a.job.dst_row = dst_row;
  a.job.cache_row = cache_row;
  a.job.src_row = src_row;
  a.job.base = base;
  a.job.skip = skip;
  const void *srcs[2] = {src0, src1}, *caches[2] = {cache0, cache1};
  void *dsts[2] = {dst0, dst1}, *stgs[2] = {stg0, stg1};
  const void *scales[2] = {scale0, scale1};
  void *sdsts[2] = {sdst0, sdst1};
  const int64_t Ws[2] = {W0, W1}, Ps[2] = {P0, P1}, SWs[2] = {SW0, SW1};
  bool vec;
  if (!fill_names(a.job, srcs, caches, dsts, stgs, Ws, Ps, scales, sdsts, SWs, compress, vec))
    return XP_EINVAL;
  // Compressed rows with a known record layout: copy only each record's used words.
  if (chunk < 0) return XP_EINVAL;
  if (compress && chunk > 0) {
    if (chunk % 8) return XP_EINVAL;
    for (int i = 0; i < 2; ++i) {
      const int64_t N = 4 * Ws[i];  // raw bytes of a row
      if (N <= 0 || N % (32 * chunk)) return XP_EINVAL;
      a.job.groups[i] = N / (32 * chunk);
    }
  }
  if (ctas < 0 || ctas > XP_MAX_COPY_CTAS) return XP_EINVAL;
  a.copy_ctas = ctas > 0 ? ctas : kDefaultCtas;
  a.fetch = req != nullptr;
  if (a.fetch) {
    if (!skip || !ring_ok(seq, req, done, block, ring) || K > block || retry_ns < 0 ||
        retry_ns > XP_MAX_RETRY_NS || giveup < 0 || giveup > XP_MAX_GIVEUP)
      return XP_EINVAL;
    a.f = Fetch{skip, K, src_row, base, layer, seq, seq, req, done, block, ring, retry_ns, giveup};
  }
  const unsigned grid = static_cast<unsigned>(a.copy_ctas + (a.fetch ? 1 : 0));
  cudaStream_t s = as_stream(stream);
  if (vec)
    gather_kernel<true><<<grid, kThreads, 0, s>>>(a);
  else
    gather_kernel<false><<<grid, kThreads, 0, s>>>(a);
  return launch_status();
}

extern "C" int xp_fetch_publish(const int64_t *todo, int64_t K, const int64_t *row_of,
                                int64_t base, int64_t layer, int64_t *seq, int64_t *ticket,
                                int64_t *req, int64_t block, int64_t ring, void *stream) {
  if (K < 0 || (K > 0 && (!todo || !row_of)) || !ticket || K > block ||
      !ring_ok(seq, req, req, block, ring))
    return XP_EINVAL;
  Fetch f{todo, K, row_of, base, layer, seq, ticket, req, nullptr, block, ring, 0, 0};
  fetch_kernel<<<1, 256, 0, as_stream(stream)>>>(f, 1, 0);
  return launch_status();
}

extern "C" int xp_fetch_wait(const int64_t *todo, int64_t K, const int64_t *ticket, int64_t *req,
                             const int64_t *done, int64_t block, int64_t ring, int64_t retry_ns,
                             int64_t giveup, void *stream) {
  if (K < 0 || (K > 0 && !todo) || !ticket || !req || !done || block < 1 || ring < 1 ||
      retry_ns < 0 || retry_ns > XP_MAX_RETRY_NS || giveup < 0 || giveup > XP_MAX_GIVEUP)
    return XP_EINVAL;
  Fetch f{todo, K, nullptr, 0, 0, nullptr, const_cast<int64_t *>(ticket), req, done, block, ring,
          retry_ns, giveup};
  fetch_kernel<<<1, 256, 0, as_stream(stream)>>>(f, 0, 1);
  return launch_status();
}

extern "C" int xp_fetch(const int64_t *todo, int64_t K, const int64_t *row_of, int64_t base,
                        int64_t layer, int64_t *seq, int64_t *req, const int64_t *done,
                        int64_t block, int64_t ring, int64_t retry_ns, int64_t giveup,
                        void *stream) {
  if (K < 0 || (K > 0 && (!todo || !row_of)) || K > block || !ring_ok(seq, req, done, block, ring) ||
      retry_ns < 0 || retry_ns > XP_MAX_RETRY_NS || giveup < 0 || giveup > XP_MAX_GIVEUP)
    return XP_EINVAL;
  // gather.py:285-287: the ticket is seq itself.
  Fetch f{todo, K, row_of, base, layer, seq, seq, req, done, block, ring, retry_ns, giveup};
  fetch_kernel<<<1, 256, 0, as_stream(stream)>>>(f, 1, 1);
  return launch_status();
}
