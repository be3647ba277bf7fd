// Device functions of the gather and of the SSD request ring, shared by
// gather.cu and step.cu.
//
// Semantics follow monochromegane/vllm-expert-pager src/vllm_expert_pager/gather.py
// (_copy_row, _copy_scale, _gather_loop, _fetch_publish, _fetch_wait).
//
// The RAM tier is pinned host memory read over the host link with 16-byte
// loads.  A few CTAs walk the (row, 16 KiB piece) units round robin so that all
// of them stay on neighbouring pieces of the same rows; each thread keeps
// kUnroll 16-byte loads in flight before storing, so the bytes in flight are
// ctas x 16 KiB.  Too many outstanding host reads queue behind each other and
// lower the link's throughput (gather.py:19-24), so the CTA count is a tuning
// argument rather than "one CTA per piece".
#pragma once

#include "common.cuh"

namespace xp {
namespace gdev {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int64_t kPieceWords = kThreads * kUnroll * 4;  // 16 KiB per unit
constexpr int kMaxK = 2048;

struct Name {
  const int32_t *src, *cache;
  int32_t *dst, *stg;
  int64_t W, P, C;  // raw words, pitch words, pieces per row
  const int32_t *scale;
  int32_t *sdst;
  int64_t SW;
};

struct Fetch {
  const int64_t *todo;  // the list to read
  int64_t K;
  const int64_t *row_of;
  int64_t base, layer;
  int64_t *seq, *ticket, *req;
  const int64_t *done;
  int64_t block, ring, retry_ns, giveup;
};

// One copy job: the gather_rows contract (gather.py:328-393).
struct CopyJob {
  const int64_t *todo;
  int64_t K;
  const int64_t *dst_row, *cache_row, *src_row;
  int64_t base;
  Name n[2];
  const int64_t *skip;   // entries listed here are not copied (may be null)
  int compress;
  // If set, the staging row of entry e is the position of e in stage_of[0:K]
  // instead of its position in todo (the fused step's SSD pass).
  const int64_t *stage_of;
  // Groups per row of each name (records of 32 x chunk values per group), or 0.
  // When set (compressed rows, at most kMaxUsed active entries), only a record's
  // used words -- header, nibbles and Huffman words, G + 1 + W/2 + header[G] --
  // cross the host link: the decoder never reads past them.
  int64_t groups[2];
};

constexpr int kMaxUsed = 64;

// Shared memory of copy_rows.
struct CopySmem {
  int list[kMaxK];       // todo positions of the active entries, in order
  int64_t skip[kMaxK];
  int count;
  int warp[kThreads / 32];
  int64_t used[kMaxUsed][2];  // words to copy of each active entry's record, per name
};

// ---- the request ring (gather.py:197-277) ----

// True on every thread if list[0:K] holds an entry >= 0 (loads bypass L1:
// the list may have been written by another CTA of the same launch).
__device__ inline bool any_entry(const int64_t *list, int64_t K) {
  __shared__ int s_any;
  if (threadIdx.x == 0) s_any = 0;
  __syncthreads();
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x)
    if (__ldcg(list + k) >= 0) s_any = 1;
  __syncthreads();
  return s_any != 0;
}

__device__ inline int64_t *ring_slot(int64_t *req, int64_t seq, int64_t ring, int64_t block) {
  return req + 2 + (seq % ring) * (2 + 2 * block);
}

// Publish the request for list[0:K] (gather.py:197-234).  The whole slot is
// written so no entry of an older request survives; seq is stored last with
// release semantics at system scope, after every thread's writes were fenced.
__device__ inline void fetch_publish(const Fetch &f) {
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
    int64_t e = i < f.K ? __ldcg(f.todo + i) : -1;
    slot[2 + i] = e;
    slot[2 + f.block + i] = e >= 0 ? __ldcg(f.row_of + e) + f.base : -1;
  }
  if (threadIdx.x == 0) slot[1] = f.layer;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) store_release_sys(slot, seq);
}

// Wait for done >= *ticket with a bounded number of re-publishes
// (gather.py:237-277).  Only req[0] and req[1] are modified, by this thread
// alone, so plain system-scope loads and stores suffice (host-link atomics on
// pinned memory are not available on every platform).  Returns on every
// thread; thread 0 did the waiting.
__device__ inline void fetch_wait(const Fetch &f) {
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

// Copy the rows and scales of the active entries of a job; this CTA takes
// units cta, cta + nctas, ... of the (entry, piece) sequence
// (gather.py:102-146).  Index arrays are read through L2 (they may come from
// another CTA of the same launch).
template <bool VEC>
__device__ void copy_rows(const CopyJob &a, int cta, int nctas, CopySmem &sm) {
  const int tid = threadIdx.x;
  if (a.skip)
    for (int64_t k = tid; k < a.K; k += kThreads) sm.skip[k] = __ldcg(a.skip + k);
  if (tid == 0) sm.count = 0;
  __syncthreads();
  // Active entries in todo order (an ordered compaction by warp ballots).
  for (int64_t base = 0; base < a.K; base += kThreads) {
    const int64_t j = base + tid;
    bool act = false;
    if (j < a.K) {
      const int64_t e = __ldcg(a.todo + j);
      act = e >= 0;
      if (act && a.skip)
        for (int64_t k = 0; k < a.K; ++k) act &= (sm.skip[k] != e);
    }
    const unsigned m = __ballot_sync(0xffffffffu, act);
    if ((tid & 31) == 0) sm.warp[tid >> 5] = __popc(m);
    __syncthreads();
    int before = sm.count;
    for (int w = 0; w < (tid >> 5); ++w) before += sm.warp[w];
    if (act) sm.list[before + __popc(m & lanemask_lt())] = static_cast<int>(j);
    __syncthreads();
    if (tid == 0) {
      int add = 0;
      for (int w = 0; w < kThreads / 32; ++w) add += sm.warp[w];
      sm.count += add;
    }
    __syncthreads();
  }
  const int64_t nact = sm.count;
  const int64_t CT = a.n[0].C + a.n[1].C;
  // Used words of each compressed record that comes from the RAM tier: one read
  // of its header's last entry per (entry, name), all in one round trip.
  const bool trim = a.compress && a.groups[0] > 0 && a.groups[1] > 0 && nact <= kMaxUsed;
  if (trim) {
    for (int64_t t = tid; t < 2 * nact; t += kThreads) {
      const int which = static_cast<int>(t & 1);
      const Name &n = a.n[which];
      const int64_t e = __ldcg(a.todo + sm.list[t >> 1]);
      int64_t w = n.P;
      if (__ldcg(a.cache_row + e) < 0) {
        const int64_t G = a.groups[which];
        const int32_t *rec = n.src + (__ldcg(a.src_row + e) + a.base) * n.P;
        const int64_t huff = __ldcg(rec + G);
        w = G + 1 + n.W / 2 + (huff > 0 ? huff : 0);
        w = w < n.P ? w : n.P;
      }
      sm.used[t >> 1][which] = w;
    }
    __syncthreads();
  }
  for (int64_t u = cta; u < nact * CT; u += nctas) {
    const int64_t j = sm.list[u / CT];
    const int64_t c = u % CT;
    const int which = c < a.n[0].C ? 0 : 1;
    const Name &n = a.n[which];
    const int64_t piece = which ? c - a.n[0].C : c;
    const int64_t e = __ldcg(a.todo + j);
    int64_t dst_row = __ldcg(a.dst_row + e);
    dst_row = dst_row > 0 ? dst_row : 0;
    const int64_t cache_row = __ldcg(a.cache_row + e);
    const int32_t *src;
    int32_t *dst;
    int64_t len;
    if (cache_row >= 0) {  // VRAM hit: raw row from the cache slab
      src = n.cache + cache_row * n.W;
      dst = n.dst + dst_row * n.W;
      len = n.W;
    } else {
      src = n.src + (__ldcg(a.src_row + e) + a.base) * n.P;
      int64_t srow = j;
      if (a.stage_of) {
        srow = 0;
        for (int64_t k = 0; k < a.K; ++k)
          if (__ldcg(a.stage_of + k) == e) srow = k;
      }
      dst = a.compress ? n.stg + srow * n.P : n.dst + dst_row * n.P;
      len = trim ? sm.used[u / CT][which] : n.P;
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

}  // namespace gdev
}  // namespace xp
