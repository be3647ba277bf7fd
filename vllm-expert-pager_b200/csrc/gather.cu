// Gather of missed expert rows into VRAM slots, and the GPU side of the SSD
// request ring.
//
// Semantics follow monochromegane/vllm-expert-pager src/vllm_expert_pager/gather.py
// (gather_rows, _fetch_publish, _fetch_wait).  The copy is done by the SMs, not
// a copy engine, so that the rows to move are read from device-resident index
// arrays and the launch can be replayed from a CUDA graph (gather.py:15-17).
//
// B200 design: the RAM tier is pinned host memory read over the host link with
// 16-byte loads.  A few CTAs walk the (row, 16 KiB piece) units round robin so
// that all CTAs stay on neighbouring pieces of the same rows; each thread keeps
// kUnroll 16-byte loads in flight before storing, so the bytes in flight are
// ctas x 16 KiB.  Too many outstanding host reads queue behind each other and
// lower the link's throughput (gather.py:19-24), so the CTA count is a tuning
// argument rather than "one CTA per piece".
#include "common.cuh"

namespace xp {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int64_t kPieceWords = kThreads * kUnroll * 4;  // 16 KiB per unit
constexpr int kMaxK = 2048;
constexpr int kDefaultCtas = 16;

struct Name {
  const int32_t *src, *cache;
  int32_t *dst, *stg;
  int64_t W, P, C;  // raw words, pitch words, pieces per row
  const int32_t *scale;
  int32_t *sdst;
  int64_t SW;
};

struct Fetch {
  const int64_t *todo;  // the list to read (the gather's skip list)
  int64_t K;
  const int64_t *row_of;
  int64_t base, layer;
  int64_t *seq, *ticket, *req;
  const int64_t *done;
  int64_t block, ring, retry_ns, giveup;
};

struct GatherArgs {
  const int64_t *todo;
  int64_t K;
  const int64_t *dst_row, *cache_row, *src_row;
  int64_t base;
  Name n[2];
  const int64_t *skip;
  int compress;
  int copy_ctas;
  int fetch;  // the last CTA runs the fetch
  Fetch f;
};

// ---- the request ring (gather.py:197-277) ----

// True on every thread if list[0:K] holds an entry >= 0.
__device__ bool any_entry(const int64_t *list, int64_t K) {
  __shared__ int s_any;
  if (threadIdx.x == 0) s_any = 0;
  __syncthreads();
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x)
    if (list[k] >= 0) s_any = 1;
  __syncthreads();
  return s_any != 0;
}

__device__ int64_t *ring_slot(int64_t *req, int64_t seq, int64_t ring, int64_t block) {
  return req + 2 + (seq % ring) * (2 + 2 * block);
}

// Publish the request for list[0:K] (gather.py:197-234).  The whole slot is
// written so no entry of an older request survives; seq is stored last with
// release semantics at system scope, after every thread's writes were fenced.
__device__ void fetch_publish(const Fetch &f) {
  if (!any_entry(f.todo, f.K)) return;
  __shared__ int64_t s_seq;
  if (threadIdx.x == 0) {
    s_seq = *f.seq + 1;
    *f.seq = s_seq;
    *f.ticket = s_seq;
  }
  __syncthreads();
  const int64_t seq = s_seq;
  int64_t *slot = ring_slot(f.req, seq, f.ring, f.block);
  for (int64_t i = threadIdx.x; i < f.block; i += blockDim.x) {
    int64_t e = i < f.K ? f.todo[i] : -1;
    slot[2 + i] = e;
    slot[2 + f.block + i] = e >= 0 ? f.row_of[e] + f.base : -1;
  }
  if (threadIdx.x == 0) slot[1] = f.layer;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) store_release_sys(slot, seq);
}

// Wait for done >= *ticket with a bounded number of re-publishes
// (gather.py:237-277).  Only req[0] and req[1] are modified, by this thread
// alone, so plain system-scope loads and stores suffice (host-link atomics on
// pinned memory are not available on every platform).
__device__ void fetch_wait(const Fetch &f) {
  if (!any_entry(f.todo, f.K)) return;
  if (threadIdx.x != 0) return;
  const int64_t seq = *f.ticket;
  int64_t *slot = ring_slot(f.req, seq, f.ring, f.block);
  int64_t d = load_acquire_sys(f.done);
  int64_t tries = 0;
  uint64_t t0 = global_ns();
  while (d < seq && tries < f.giveup) {
    uint64_t now = global_ns();
    if (now - t0 >= static_cast<uint64_t>(f.retry_ns)) {
      // Still waiting: publish again and count it, so a lost handoff in
      // either direction recovers (the host rewrites done when req[0] moves).
      t0 = now;
      ++tries;
      store_release_sys(slot, seq);
      store_release_sys(f.req, load_relaxed_sys(f.req) + 1);
    }
    __nanosleep(256);
    d = load_acquire_sys(f.done);
  }
  if (d < seq) store_release_sys(f.req + 1, load_relaxed_sys(f.req + 1) + 1);
}

__global__ void fetch_kernel(const __grid_constant__ Fetch f, int publish, int wait) {
  if (publish) fetch_publish(f);
  if (publish && wait) __syncthreads();
  if (wait) fetch_wait(f);
}

// ---- the copy ----

template <bool VEC>
__device__ __forceinline__ void copy_piece(const int32_t *__restrict__ src, int32_t *__restrict__ dst,
                                           int64_t words) {
  if (VEC) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    const int64_t nv = words / 4;
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      int64_t i = threadIdx.x + u * kThreads;
      if (i < nv) v[u] = __ldcg(s + i);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      int64_t i = threadIdx.x + u * kThreads;
      if (i < nv) d[i] = v[u];
    }
    for (int64_t w = nv * 4 + threadIdx.x; w < words; w += kThreads) dst[w] = __ldcg(src + w);
  } else {
    for (int64_t w = threadIdx.x; w < words; w += kThreads) dst[w] = __ldcg(src + w);
  }
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
  __shared__ int s_list[kMaxK];   // todo indices j of the active entries, in order
  __shared__ int64_t s_skip[kMaxK];
  __shared__ int s_count;
  const int tid = threadIdx.x;
  if (a.skip)
    for (int64_t k = tid; k < a.K; k += kThreads) s_skip[k] = a.skip[k];
  if (tid == 0) s_count = 0;
  __syncthreads();
  // Active entries in todo order (an ordered compaction by warp ballots).
  for (int64_t base = 0; base < a.K; base += kThreads) {
    int64_t j = base + tid;
    bool act = false;
    if (j < a.K) {
      int64_t e = a.todo[j];
      act = e >= 0;
      if (act && a.skip)
        for (int64_t k = 0; k < a.K; ++k) act &= (s_skip[k] != e);
    }
    __shared__ int s_warp[kThreads / 32];
    unsigned m = __ballot_sync(0xffffffffu, act);
    if ((tid & 31) == 0) s_warp[tid >> 5] = __popc(m);
    __syncthreads();
    int before = s_count;
    for (int w = 0; w < (tid >> 5); ++w) before += s_warp[w];
    if (act) s_list[before + __popc(m & lanemask_lt())] = static_cast<int>(j);
    __syncthreads();
    if (tid == 0) {
      int add = 0;
      for (int w = 0; w < kThreads / 32; ++w) add += s_warp[w];
      s_count += add;
    }
    __syncthreads();
  }
  const int64_t nact = s_count;
  const int64_t CT = a.n[0].C + a.n[1].C;
  for (int64_t u = blockIdx.x; u < nact * CT; u += a.copy_ctas) {
    const int64_t j = s_list[u / CT];
    const int64_t c = u % CT;
    const int which = c < a.n[0].C ? 0 : 1;
    const Name &n = a.n[which];
    const int64_t piece = which ? c - a.n[0].C : c;
    const int64_t e = a.todo[j];
    int64_t dst_row = a.dst_row[e];
    dst_row = dst_row > 0 ? dst_row : 0;
    const int64_t cache_row = a.cache_row[e];
    const int32_t *src;
    int32_t *dst;
    int64_t len;
    if (cache_row >= 0) {  // VRAM hit: raw row from the cache slab
      src = n.cache + cache_row * n.W;
      dst = n.dst + dst_row * n.W;
      len = n.W;
    } else {
      src = n.src + (a.src_row[e] + a.base) * n.P;
      dst = a.compress ? n.stg + j * n.P : n.dst + dst_row * n.P;
      len = n.P;
    }
    const int64_t off = piece * kPieceWords;
    if (off < len) {
      int64_t words = len - off < kPieceWords ? len - off : kPieceWords;
      copy_piece<VEC>(src + off, dst + off, words);
    }
    if (piece == 0)  // the scale row follows the weights into the slot
      for (int64_t w = tid; w < n.SW; w += kThreads)
        n.sdst[dst_row * n.SW + w] = n.scale[e * n.SW + w];
  }
}

}  // namespace
}  // namespace xp

using namespace xp;

namespace {

bool ring_ok(const int64_t *seq, const int64_t *req, const int64_t *done, int64_t block,
             int64_t ring) {
  return seq && req && done && block >= 1 && ring >= 1;
}

}  // namespace

extern "C" int xp_gather_rows(const int64_t *todo, int64_t K, const int64_t *dst_row,
                              const int64_t *cache_row, const int64_t *src_row, int64_t base,
                              const void *src0, const void *cache0, void *dst0, void *stg0,
                              int64_t W0, int64_t P0, const void *src1, const void *cache1,
                              void *dst1, void *stg1, int64_t W1, int64_t P1, const void *scale0,
                              void *sdst0, int64_t SW0, const void *scale1, void *sdst1,
                              int64_t SW1, const int64_t *skip, int compress, int ctas,
                              int64_t layer, int64_t *seq, int64_t *req, const int64_t *done,
                              int64_t block, int64_t ring, int64_t retry_ns, int64_t giveup,
                              void *stream) {
  if (K < 0 || K > kMaxK || (K > 0 && (!todo || !dst_row || !cache_row || !src_row)))
    return XP_EINVAL;
  if (W0 < 0 || W1 < 0 || P0 < 0 || P1 < 0 || SW0 < 0 || SW1 < 0) return XP_EINVAL;
  if (!compress && (P0 != W0 || P1 != W1)) return XP_EINVAL;
  if (compress && (!stg0 || !stg1)) return XP_EINVAL;
  if (!dst0 || !dst1 || !scale0 || !scale1 || !sdst0 || !sdst1) return XP_EINVAL;
  GatherArgs a{};
  a.todo = todo;
  a.K = K;
  a.dst_row = dst_row;
  a.cache_row = cache_row;
  a.src_row = src_row;
  a.base = base;
  const void *srcs[2] = {src0, src1}, *caches[2] = {cache0, cache1};
  void *dsts[2] = {dst0, dst1}, *stgs[2] = {stg0, stg1};
  const void *scales[2] = {scale0, scale1};
  void *sdsts[2] = {sdst0, sdst1};
  const int64_t Ws[2] = {W0, W1}, Ps[2] = {P0, P1}, SWs[2] = {SW0, SW1};
  bool vec = true;
  for (int i = 0; i < 2; ++i) {
    Name &n = a.n[i];
    n.src = static_cast<const int32_t *>(srcs[i]);
    n.cache = static_cast<const int32_t *>(caches[i]);
    n.dst = static_cast<int32_t *>(dsts[i]);
    n.stg = static_cast<int32_t *>(stgs[i]);
    n.W = Ws[i];
    n.P = Ps[i];
    int64_t m = Ws[i] > Ps[i] ? Ws[i] : Ps[i];
    n.C = (m + kPieceWords - 1) / kPieceWords;
    n.scale = static_cast<const int32_t *>(scales[i]);
    n.sdst = static_cast<int32_t *>(sdsts[i]);
    n.SW = SWs[i];
    vec = vec && (Ws[i] % 4 == 0) && (Ps[i] % 4 == 0) && aligned(srcs[i], 16) &&
          aligned(caches[i], 16) && aligned(dsts[i], 16) && (!compress || aligned(stgs[i], 16));
  }
  a.skip = skip;
  a.compress = compress;
  a.copy_ctas = ctas > 0 ? ctas : kDefaultCtas;
  a.fetch = req != nullptr;
  if (a.fetch) {
    if (!skip || !ring_ok(seq, req, done, block, ring) || K > block || retry_ns < 0 || giveup < 0)
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
      retry_ns < 0 || giveup < 0)
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
      retry_ns < 0 || giveup < 0)
    return XP_EINVAL;
  // gather.py:285-287: the ticket is seq itself.
  Fetch f{todo, K, row_of, base, layer, seq, seq, req, done, block, ring, retry_ns, giveup};
  fetch_kernel<<<1, 256, 0, as_stream(stream)>>>(f, 1, 1);
  return launch_status();
}
