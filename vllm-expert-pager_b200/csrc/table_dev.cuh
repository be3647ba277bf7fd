// Device functions of the slot-table kernels, shared by table.cu and step.cu.
//
// Semantics follow monochromegane/vllm-expert-pager src/vllm_expert_pager/table.py
// (ExpertTable); citations per function.
#pragma once

#include <cub/block/block_scan.cuh>

#include "common.cuh"

namespace xp {
namespace tdev {

constexpr int kThreads = 256;
// Pushes slots whose expert is used this step to the end of the victim order
// (table.py:14-16).
constexpr unsigned long long kProtect = 1ull << 40;

using BlockScan = cub::BlockScan<int, kThreads, cub::BLOCK_SCAN_WARP_SCANS>;

// Shared memory of one table update.  Each table is read from global memory
// once, with coalesced loads, into slot/occ/key; the update then works on
// these copies and writes back only what changes.
struct TableSmem {
  long long *step;            // the table's step counter
  uint8_t *need;              // [E] experts needed this step
  int *rank;                  // [E] ordinal of a miss, -1 otherwise
  int *slot;                  // [E] slot_of (kept up to date through the update)
  unsigned long long *key;    // [S] victim key
  int *order;                 // [S] the first `misses` slots sorted by (key, slot)
  int *evic;                  // [S] expert evicted by the miss of ordinal r
  int *occ;                   // [S] expert_in before the update
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

__host__ __device__ inline size_t table_smem_bytes(int64_t E, int64_t S) {
  return 16 + 8 * S + 2 * align16(4 * E) + 3 * align16(4 * S) + align16(E);
}

__device__ inline TableSmem carve(unsigned char *base, int64_t E, int64_t S) {
  TableSmem t;
  unsigned char *p = base;
  t.step = reinterpret_cast<long long *>(p);
  p += 16;
  t.key = reinterpret_cast<unsigned long long *>(p);
  p += 8 * S;
  t.rank = reinterpret_cast<int *>(p);
  p += align16(4 * E);
  t.slot = reinterpret_cast<int *>(p);
  p += align16(4 * E);
  t.order = reinterpret_cast<int *>(p);
  p += align16(4 * S);
  t.evic = reinterpret_cast<int *>(p);
  p += align16(4 * S);
  t.occ = reinterpret_cast<int *>(p);
  p += align16(4 * S);
  t.need = p;
  return t;
}

struct Table {
  int64_t *slot_of, *expert_in, *last_used, *counters;
  int64_t slots;
};

// Copy of the table into shared memory (no barrier).  Each thread's first
// elements are loaded into registers before any shared store, so that their
// global loads are in flight together (the shared arrays are reached through
// generic pointers, which the compiler cannot tell apart from global ones).
__device__ inline void load_table(const TableSmem &sm, Table t, int64_t E) {
  const int tid = threadIdx.x;
  const int64_t S = t.slots;
  const int64_t occ0 = tid < S ? t.expert_in[tid] : 0;
  const int64_t key0 = tid < S ? t.last_used[tid] : 0;
  const int64_t slot0 = tid < E ? t.slot_of[tid] : 0;
  const int64_t step0 = tid == 0 ? t.counters[0] : 0;
  if (tid == 0) *sm.step = step0;
  if (tid < S) {
    sm.occ[tid] = static_cast<int>(occ0);
    sm.key[tid] = static_cast<unsigned long long>(key0);
  }
  if (tid < E) sm.slot[tid] = static_cast<int>(slot0);
  for (int64_t s = tid + kThreads; s < S; s += kThreads) {
    sm.occ[s] = static_cast<int>(t.expert_in[s]);
    sm.key[s] = static_cast<unsigned long long>(t.last_used[s]);
  }
  for (int64_t e = tid + kThreads; e < E; e += kThreads) sm.slot[e] = static_cast<int>(t.slot_of[e]);
}

// need[e] = e occurs in ids[0:K] (table.py:63-71) and the table copy, with the
// ids and the table loaded from global memory in one round trip.  Ends with a
// barrier.
__device__ inline void need_and_table(const TableSmem &sm, Table t, const void *ids,
                                      int ids_bytes, int64_t K, int64_t E) {
  const int tid = threadIdx.x;
  const int64_t id0 = tid < K ? load_id(ids, ids_bytes, tid) : -1;
  load_table(sm, t, E);
  for (int64_t e = tid; e < E; e += kThreads) sm.need[e] = 0;
  __syncthreads();
  if (id0 >= 0 && id0 < E) sm.need[id0] = 1;
  for (int64_t k = tid + kThreads; k < K; k += kThreads) {
    const int64_t id = load_id(ids, ids_bytes, k);
    if (id >= 0 && id < E) sm.need[id] = 1;
  }
  __syncthreads();
}

// ExpertTable.acquire (table.py:75-128) given the need mask in shared memory;
// `loaded`: the table copy is already in shared memory (need_and_table).
//
// Victims: slots in ascending order of last_used + PROTECT*used, ties by slot
// number (the stable argsort of table.py:107-108); the miss of ordinal r (misses
// in ascending expert id, table.py:109) takes the r-th slot of that order, so
// only the first `misses` positions of the order are computed, and none when
// every needed expert hits.  The slot outputs read slot_of after the update, as
// the torch version does (table.py:95,118).  Outputs may be null.  count: add
// hits/misses to the counters (seed restores them, table.py:170-171).
__device__ inline void acquire_table(const TableSmem &sm, Table t, int64_t E, int64_t K,
                                     int32_t *map32, int64_t *map64, int64_t *slot_out,
                                     int64_t *todo, bool count, bool loaded) {
  const int tid = threadIdx.x;
  const int64_t S = t.slots;
  __shared__ typename BlockScan::TempStorage scan_tmp;

  if (!loaded) {
    load_table(sm, t, E);
    __syncthreads();
  }
  const int64_t step = *sm.step;
  // Victim keys: slots whose expert is used this step go last (table.py:100-107).
  for (int64_t s = tid; s < S; s += kThreads) {
    const int occ = sm.occ[s];
    if (occ >= 0 && occ < E && sm.need[occ] && sm.slot[occ] >= 0) sm.key[s] += kProtect;
  }
  // Hits and misses (table.py:96-97) in one scan: misses count in the low 16
  // bits, hits in the high 16 (E <= 4096); miss ordinals in ascending expert id
  // (table.py:109) over experts held in contiguous ranges per thread.
  const int64_t ipt = (E + kThreads - 1) / kThreads;
  const int64_t e0 = tid * ipt, e1 = e0 + ipt < E ? e0 + ipt : E;
  int packed = 0;
  for (int64_t e = e0; e < e1; ++e)
    if (sm.need[e]) packed += sm.slot[e] >= 0 ? 0x10000 : 1;
  int base, total;
  BlockScan(scan_tmp).ExclusiveSum(packed, base, total);
  const int misses = total & 0xFFFF, hits = total >> 16;
  {
    int r = base & 0xFFFF;
    for (int64_t e = e0; e < e1; ++e) sm.rank[e] = (sm.need[e] && sm.slot[e] < 0) ? r++ : -1;
  }
  __syncthreads();  // keys and rank[] complete
  if (misses > 0) {
    // Stable rank of every slot by its key; positions below `misses` are kept.
    for (int64_t s = tid; s < S; s += kThreads) {
      const unsigned long long k = sm.key[s];
      int pos = 0;
      for (int64_t u = 0; u < S; ++u) {
        const unsigned long long ku = sm.key[u];
        pos += (ku < k) | ((ku == k) & (u < s));
      }
      if (pos < misses) sm.order[pos] = static_cast<int>(s);
    }
    __syncthreads();
    // The expert each victim slot holds now (table.py:113).
    for (int r = tid; r < misses; r += kThreads) sm.evic[r] = sm.occ[sm.order[r < S ? r : S - 1]];
    __syncthreads();
  }

  // Update the table (table.py:114-120).  The experts written here are
  // disjoint: evicted experts are cached and not needed; misses are not cached.
  for (int64_t e = e0; e < e1; ++e) {
    if (!sm.need[e]) continue;
    const int r = sm.rank[e];
    if (r >= 0) {
      const int v = sm.order[r < S ? r : S - 1];
      const int ev = sm.evic[r];
      if (ev >= 0) {
        t.slot_of[ev] = -1;
        sm.slot[ev] = -1;
      }
      t.slot_of[e] = v;
      sm.slot[e] = v;
      t.expert_in[v] = e;
      t.last_used[v] = step;
      if (todo) todo[r] = e;  // table.py:126-127
    } else {
      t.last_used[sm.slot[e]] = step;
    }
  }
  if (todo)
    for (int64_t k = misses + tid; k < K; k += kThreads) todo[k] = -1;
  __syncthreads();  // slot[] updated
  for (int64_t e = tid; e < E; e += kThreads) {
    const int64_t s = sm.slot[e];  // slot_of after the update (table.py:95,118)
    if (slot_out) slot_out[e] = s;
    const int64_t m = sm.need[e] ? s : -1;  // table.py:125
    if (map32) map32[e] = static_cast<int32_t>(m);
    if (map64) map64[e] = m;
  }
  if (tid == 0) {
    t.counters[0] = step + 1;
    if (count) {
      t.counters[1] += hits;
      t.counters[2] += misses;
    }
  }
  __syncthreads();
}

}  // namespace tdev
}  // namespace xp
