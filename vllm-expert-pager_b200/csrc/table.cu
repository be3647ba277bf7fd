// Slot-table kernels: acquire (one table or the VRAM/RAM pair), need_mask, seed,
// plan_chunks.
//
// Semantics follow monochromegane/vllm-expert-pager src/vllm_expert_pager/table.py
// (ExpertTable) and acquire.py (the fused pair); citations per function.  One
// CTA owns one table: the work is a few hundred integers, so the kernel is
// latency-bound, and a single CTA keeps every phase ordered by __syncthreads
// instead of global atomics or extra launches.
#include "table_dev.cuh"

namespace xp {
namespace {

using namespace tdev;

struct PairArgs {
  const void *ids;
  int ids_bytes;
  int64_t K, E;
  Table a, b;
  int32_t *map32;
  int64_t *a_slot, *a_todo, *b_slot, *b_todo;
};

// acquire.py:103-141: CTA 0 updates the VRAM table and writes expert_map, CTA 1
// the RAM table.
__global__ void __launch_bounds__(kThreads) acquire_pair_kernel(const __grid_constant__ PairArgs p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int64_t S = p.a.slots > p.b.slots ? p.a.slots : p.b.slots;
  TableSmem sm = carve(smem, p.E, S);
  // One code path for both CTAs (half the instruction footprint of two inlined
  // copies): the CTA index selects the table and its outputs.
  const bool vram = blockIdx.x == 0;
  const Table t = vram ? p.a : p.b;
  need_and_table(sm, t, p.ids, p.ids_bytes, p.K, p.E);
  acquire_table(sm, t, p.E, p.K, vram ? p.map32 : nullptr, nullptr, vram ? p.a_slot : p.b_slot,
                vram ? p.a_todo : p.b_todo, true, true);
}

struct OneArgs {
  const void *ids;
  int ids_bytes;
  int64_t K, E;
  Table t;
  int64_t *map64, *slot, *todo;
};

__global__ void __launch_bounds__(kThreads) acquire_kernel(const __grid_constant__ OneArgs p) {
  extern __shared__ __align__(16) unsigned char smem[];
  TableSmem sm = carve(smem, p.E, p.t.slots);
  need_and_table(sm, p.t, p.ids, p.ids_bytes, p.K, p.E);
  acquire_table(sm, p.t, p.E, p.K, nullptr, p.map64, p.slot, p.todo, true, true);
}

__global__ void need_mask_kernel(const void *ids, int ids_bytes, int64_t K, int64_t E,
                                 uint8_t *need) {
  // Pass 1 of need_mask: clear; need_scatter_kernel then sets the ids present.
  for (int64_t e = blockIdx.x * blockDim.x + threadIdx.x; e < E;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x)
    need[e] = 0;
}

__global__ void need_scatter_kernel(const void *ids, int ids_bytes, int64_t K, int64_t E,
                                    uint8_t *need) {
  for (int64_t k = blockIdx.x * blockDim.x + threadIdx.x; k < K;
       k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t id = load_id(ids, ids_bytes, k);
    if (id >= 0 && id < E) need[id] = 1;
  }
}

struct SeedArgs {
  const void *ids;
  int ids_bytes;
  int64_t K, E;
  Table t;  // the RAM table (R slots)
  const int64_t *vram_expert_in;
  int64_t S;
  const uint8_t *need;
  const int64_t *top_in;
  int64_t *top_out;
};

// ExpertTable.seed (table.py:140-171), run by one CTA with table_smem_bytes(E, R)
// + 4E + 4*max(R-S,1) bytes of shared memory at smem.
__device__ void seed_body(const SeedArgs &p, unsigned char *smem) {
  const int64_t E = p.E, R = p.t.slots, S = p.S;
  const int64_t ntop = R - S > 1 ? R - S : 1;
  TableSmem sm = carve(smem, E, R);
  // Extra shared arrays after the table's: counts[E], top[ntop].
  int *counts = reinterpret_cast<int *>(smem + table_smem_bytes(E, R));
  int *top = counts + E;
  const int tid = threadIdx.x;

  // Reference counts (table.py:155-160).
  for (int64_t e = tid; e < E; e += kThreads) counts[e] = 0;
  __syncthreads();
  for (int64_t k = tid; k < p.K; k += kThreads) {
    int64_t id = load_id(p.ids, p.ids_bytes, k);
    if (id >= 0 && id < E) atomicAdd(&counts[id], 1);
  }
  __syncthreads();
  // The ntop most referenced experts, ties by lower id (table.py:161).
  if (p.top_in) {
    for (int64_t i = tid; i < ntop; i += kThreads) top[i] = static_cast<int>(p.top_in[i]);
  } else {
    for (int64_t e = tid; e < E; e += kThreads) {
      const int c = counts[e];
      int64_t pos = 0;
      for (int64_t u = 0; u < E; ++u) {
        int cu = counts[u];
        pos += (cu > c) | ((cu == c) & (u < e));
      }
      if (pos < ntop) top[pos] = static_cast<int>(e);
    }
  }
  __syncthreads();
  const int top0 = top[0];
  // Unreferenced entries become the first one (table.py:164).
  for (int64_t i = tid; i < ntop; i += kThreads) {
    int x = top[i];
    int y = counts[x] > 0 ? x : top0;
    if (p.top_out) p.top_out[i] = y;
    top[i] = y;
  }
  __syncthreads();
  if (R > S) {  // table.py:165-166
    for (int64_t e = tid; e < E; e += kThreads) sm.need[e] = 0;
    __syncthreads();
    for (int64_t i = tid; i < ntop; i += kThreads) sm.need[top[i]] = 1;
    __syncthreads();
    acquire_table(sm, p.t, E, ntop, nullptr, nullptr, nullptr, nullptr, false, false);
  }
  // The VRAM tier's experts that are in the RAM table or referenced
  // (table.py:167-169).
  for (int64_t e = tid; e < E; e += kThreads) sm.need[e] = 0;
  __syncthreads();
  for (int64_t s = tid; s < S; s += kThreads) {
    int64_t v = p.vram_expert_in[s];
    bool ok = v >= 0 && v < E && (p.t.slot_of[v] >= 0 || p.need[v]);
    sm.need[ok ? v : top0] = 1;
  }
  __syncthreads();
  acquire_table(sm, p.t, E, S, nullptr, nullptr, nullptr, nullptr, false, false);
}

__global__ void __launch_bounds__(kThreads) seed_kernel(const __grid_constant__ SeedArgs p) {
  extern __shared__ __align__(16) unsigned char smem[];
  seed_body(p, smem);
}

struct PlanArgs {
  int64_t E;
  const int64_t *slot_of, *before;
  const uint8_t *need;
  const int64_t *cached_row;
  int64_t W, ram_base, working_base;
  int64_t *dst_row, *src_row, *maps, *todo, *ssd, *late;
};

// ExpertTable.plan_chunks (table.py:173-247), run by one CTA.
__device__ void plan_body(const PlanArgs &p) {
  __shared__ typename BlockScan::TempStorage tmp_a, tmp_b;
  const int tid = threadIdx.x;
  const int64_t E = p.E, W = p.W, N = (E + W - 1) / W + 1, NW = N * W;
  const int64_t ipt = (E + kThreads - 1) / kThreads;
  const int64_t e0 = tid * ipt, e1 = e0 + ipt < E ? e0 + ipt : E;

  // Experts whose old RAM slot is still usable need no SSD wait (table.py:214-216).
  int na = 0, nb = 0;
  for (int64_t e = e0; e < e1; ++e) {
    int64_t before = p.before[e], after = p.slot_of[e];
    bool need = p.need[e];
    bool old_ok = before >= 0 && (after < 0 || after == before);
    bool ssd = !old_ok && (need || before >= 0);
    na += need && !ssd;
    nb += ssd;
  }
  int abase, atot, bbase, btot;
  BlockScan(tmp_a).ExclusiveSum(na, abase, atot);
  BlockScan(tmp_b).ExclusiveSum(nb, bbase, btot);
  // The SSD group starts at the next chunk boundary (table.py:219).
  const int64_t boundary = (atot + W - 1) / W * W;

  for (int64_t i = tid; i < NW; i += kThreads) {
    p.todo[i] = -1;
    p.ssd[i] = -1;
    p.late[i] = -1;
  }
  __syncthreads();
  int64_t a = abase, b = bbase;
  for (int64_t e = e0; e < e1; ++e) {
    int64_t before = p.before[e], after = p.slot_of[e];
    bool need = p.need[e];
    bool old_ok = before >= 0 && (after < 0 || after == before);
    bool ssd = !old_ok && (need || before >= 0);
    bool first = need && !ssd;
    a += first;
    b += ssd;
    int64_t pos = first ? a - 1 : boundary + b - 1;  // table.py:220
    int64_t dst = floor_mod(pos, W);
    int64_t q = floor_div(pos, W);
    int64_t shared = p.working_base + floor_mod(q, 2) * W + dst;
    p.dst_row[e] = dst;
    p.src_row[e] = old_ok ? before + p.ram_base : (after >= 0 ? after + p.ram_base : shared);
    int64_t chunk = need ? q : -1;
    for (int64_t k = 0; k < N; ++k) p.maps[k * E + e] = chunk == k ? dst : -1;
    // table.py:235-247
    bool cached = p.cached_row[e] >= 0;
    if (need && (!ssd || cached)) p.todo[pos] = e;
    if (ssd) p.ssd[pos] = e;
    if (need && ssd && !cached) p.late[pos] = e;
  }
}

__global__ void __launch_bounds__(kThreads) plan_kernel(const __grid_constant__ PlanArgs p) {
  plan_body(p);
}

struct WorkArgs {
  const void *ids;
  int ids_bytes;
  int64_t K, E;
  Table t;  // the RAM table (R slots)
  const int64_t *vram_expert_in, *cached_row;
  int64_t S, W, ram_base, working_base;
  const int64_t *top_in;
  int64_t *top_out;
  uint8_t *need;
  int64_t *before, *dst_row, *src_row, *maps, *todo, *ssd, *late;
};

// The planning of one working-path step (experts.py:500-511) in one CTA:
// need_mask, the copy of slot_of, acquire (K <= R) or seed, plan_chunks.
__global__ void __launch_bounds__(kThreads) plan_working_kernel(const __grid_constant__ WorkArgs p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x;
  const int64_t E = p.E, R = p.t.slots;
  for (int64_t e = tid; e < E; e += kThreads) {
    p.need[e] = 0;
    p.before[e] = p.t.slot_of[e];
  }
  __syncthreads();
  for (int64_t k = tid; k < p.K; k += kThreads) {
    const int64_t id = load_id(p.ids, p.ids_bytes, k);
    if (id >= 0 && id < E) p.need[id] = 1;
  }
  __syncthreads();
  if (p.K <= R) {  // ram.acquire(topk_ids): hits and misses are counted
    TableSmem sm = carve(smem, E, R);
    for (int64_t e = tid; e < E; e += kThreads) sm.need[e] = p.need[e];
    __syncthreads();
    acquire_table(sm, p.t, E, p.K, nullptr, nullptr, nullptr, nullptr, true, false);
  } else {
    const SeedArgs sa{p.ids, p.ids_bytes, p.K, E, p.t, p.vram_expert_in, p.S, p.need,
                      p.top_in, p.top_out};
    seed_body(sa, smem);
  }
  __syncthreads();
  const PlanArgs pa{E, p.t.slot_of, p.before, p.need, p.cached_row, p.W, p.ram_base,
                    p.working_base, p.dst_row, p.src_row, p.maps, p.todo, p.ssd, p.late};
  plan_body(pa);
}

bool ids_ok(const void *ids, int ids_bytes, int64_t K) {
  return (ids_bytes == 4 || ids_bytes == 8) && K >= 0 && (ids != nullptr || K == 0);
}

bool table_ok(const Table &t, int64_t E) {
  return t.slot_of && t.expert_in && t.last_used && t.counters && t.slots >= 1 &&
         t.slots <= XP_MAX_SLOTS && E >= 1 && E <= XP_MAX_EXPERTS;
}

int set_smem(const void *fn, size_t bytes) {
  if (bytes > 48 * 1024) {
    cudaError_t err =
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (err != cudaSuccess) return static_cast<int>(err);
  }
  return XP_OK;
}

}  // namespace
}  // namespace xp

using namespace xp;

extern "C" int xp_acquire_pair(const void *ids, int ids_bytes, int64_t K, int64_t E,
                               int64_t *a_slot_of, int64_t *a_expert_in, int64_t *a_last_used,
                               int64_t *a_counters, int64_t a_slots, int32_t *expert_map,
                               int64_t *a_slot, int64_t *a_todo, int64_t *b_slot_of,
                               int64_t *b_expert_in, int64_t *b_last_used, int64_t *b_counters,
                               int64_t b_slots, int64_t *b_slot, int64_t *b_todo, void *stream) {
  PairArgs p{ids, ids_bytes, K, E,
             Table{a_slot_of, a_expert_in, a_last_used, a_counters, a_slots},
             Table{b_slot_of, b_expert_in, b_last_used, b_counters, b_slots},
             expert_map, a_slot, a_todo, b_slot, b_todo};
  if (!ids_ok(ids, ids_bytes, K) || !table_ok(p.a, E) || !table_ok(p.b, E)) return XP_EINVAL;
  if (K > a_slots || K > b_slots) return XP_EINVAL;
  const int64_t S = a_slots > b_slots ? a_slots : b_slots;
  const size_t smem = table_smem_bytes(E, S);
  int rc = set_smem((const void *)acquire_pair_kernel, smem);
  if (rc) return rc;
  acquire_pair_kernel<<<2, kThreads, smem, as_stream(stream)>>>(p);
  return launch_status();
}

extern "C" int xp_acquire(const void *ids, int ids_bytes, int64_t K, int64_t E, int64_t *slot_of,
                          int64_t *expert_in, int64_t *last_used, int64_t *counters, int64_t slots,
                          int64_t *expert_map, int64_t *slot, int64_t *todo, void *stream) {
  OneArgs p{ids, ids_bytes, K, E, Table{slot_of, expert_in, last_used, counters, slots},
            expert_map, slot, todo};
  if (!ids_ok(ids, ids_bytes, K) || !table_ok(p.t, E) || K > slots) return XP_EINVAL;
  const size_t smem = table_smem_bytes(E, slots);
  int rc = set_smem((const void *)acquire_kernel, smem);
  if (rc) return rc;
  acquire_kernel<<<1, kThreads, smem, as_stream(stream)>>>(p);
  return launch_status();
}

extern "C" int xp_need_mask(const void *ids, int ids_bytes, int64_t K, int64_t E, uint8_t *need,
                            void *stream) {
  if (!ids_ok(ids, ids_bytes, K) || !need || E < 1) return XP_EINVAL;
  cudaStream_t s = as_stream(stream);
  need_mask_kernel<<<(unsigned)((E + 255) / 256), 256, 0, s>>>(ids, ids_bytes, K, E, need);
  if (K > 0)
    need_scatter_kernel<<<(unsigned)((K + 255) / 256 < 1024 ? (K + 255) / 256 : 1024), 256, 0, s>>>(
        ids, ids_bytes, K, E, need);
  return launch_status();
}

extern "C" int xp_seed(const void *ids, int ids_bytes, int64_t K, int64_t E, int64_t *slot_of,
                       int64_t *expert_in, int64_t *last_used, int64_t *counters, int64_t R,
                       const int64_t *vram_expert_in, int64_t S, const uint8_t *need,
                       const int64_t *top_in, int64_t *top_out, void *stream) {
  SeedArgs p{ids, ids_bytes, K, E, Table{slot_of, expert_in, last_used, counters, R},
             vram_expert_in, S, need, top_in, top_out};
  if (!ids_ok(ids, ids_bytes, K) || !table_ok(p.t, E) || !vram_expert_in || !need) return XP_EINVAL;
  if (S < 1 || S > R) return XP_EINVAL;
  const int64_t ntop = R - S > 1 ? R - S : 1;
  const size_t smem = table_smem_bytes(E, R) + 4 * E + 4 * ntop;
  int rc = set_smem((const void *)seed_kernel, smem);
  if (rc) return rc;
  seed_kernel<<<1, kThreads, smem, as_stream(stream)>>>(p);
  return launch_status();
}

extern "C" int xp_plan_chunks(int64_t E, const int64_t *slot_of, const int64_t *before,
                              const uint8_t *need, const int64_t *cached_row, int64_t W,
                              int64_t ram_base, int64_t working_base, int64_t *dst_row,
                              int64_t *src_row, int64_t *maps, int64_t *todo, int64_t *ssd,
                              int64_t *late, void *stream) {
  if (E < 1 || E > XP_MAX_EXPERTS || W < 1 || !slot_of || !before || !need || !cached_row ||
      !dst_row || !src_row || !maps || !todo || !ssd || !late)
    return XP_EINVAL;
  PlanArgs p{E, slot_of, before, need, cached_row, W, ram_base, working_base,
             dst_row, src_row, maps, todo, ssd, late};
  plan_kernel<<<1, kThreads, 0, as_stream(stream)>>>(p);
  return launch_status();
}

extern "C" int xp_plan_working(const void *ids, int ids_bytes, int64_t K, int64_t E,
                               int64_t *slot_of, int64_t *expert_in, int64_t *last_used,
                               int64_t *counters, int64_t R, const int64_t *vram_expert_in,
                               const int64_t *cached_row, int64_t S, int64_t W,
                               int64_t ram_base, int64_t working_base, const int64_t *top_in,
                               int64_t *top_out, uint8_t *need, int64_t *before,
                               int64_t *dst_row, int64_t *src_row, int64_t *maps, int64_t *todo,
                               int64_t *ssd, int64_t *late, void *stream) {
  WorkArgs p{ids, ids_bytes, K, E, Table{slot_of, expert_in, last_used, counters, R},
             vram_expert_in, cached_row, S, W, ram_base, working_base, top_in, top_out,
             need, before, dst_row, src_row, maps, todo, ssd, late};
  if (!ids_ok(ids, ids_bytes, K) || !table_ok(p.t, E) || !vram_expert_in || !cached_row ||
      !need || !before || !dst_row || !src_row || !maps || !todo || !ssd || !late)
    return XP_EINVAL;
  if (S < 1 || S > R || W < 1) return XP_EINVAL;
  const int64_t ntop = R - S > 1 ? R - S : 1;
  const size_t smem = table_smem_bytes(E, R) + 4 * E + 4 * ntop;
  int rc = set_smem((const void *)plan_working_kernel, smem);
  if (rc) return rc;
  plan_working_kernel<<<1, kThreads, smem, as_stream(stream)>>>(p);
  return launch_status();
}
