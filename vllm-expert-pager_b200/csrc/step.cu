// One launch for the paging of a decode step: xp_decode_step.
//
// The reference pages a decode step with three launches on one stream
// (experts.py:406-447): the table update of both tiers (acquire.py), a gather
// whose last CTA also asks the host for the SSD misses and waits
// (gather.py:149-194), and a second gather for the rows the host read.  Here
// one grid does all of it:
//   CTA 0, 1        update the VRAM and RAM tables (table_dev.cuh), then raise
//                   the "tables" flag;
//   CTA 2 .. 2+C-1  wait for the flag, copy the misses that are in RAM
//                   (gather_dev.cuh), wait for the "ssd" flag, copy the rows the
//                   host read (compressed rows go to the staging row of their
//                   position in the VRAM miss list, so one decode launch after
//                   this one expands every miss);
//   last CTA        (when there is an SSD tier) waits for the tables, publishes
//                   the request, waits for the host, raises the "ssd" flag.
// The grid is a few dozen CTAs; the launch is refused (XP_ERANGE) unless all of
// them fit on the GPU at once (occupancy x SM count), so the waiting CTAs never
// hold the SMs that the CTAs they wait for need.  Every wait is bounded: after
// its limit a CTA gives up, counts an error in scratch[3] (and, if the caller
// gave one, writes the new count to errors_out) and skips its work.
// The scratch block (XP_STEP_SCRATCH_BYTES) holds the flags and a finished
// counter; the last CTA to finish clears them, so every launch starts from
// zero and the launch replays from a CUDA graph.
#include <atomic>
#include <mutex>

#include "gather_dev.cuh"
#include "table_dev.cuh"

namespace xp {

bool fill_names(gdev::CopyJob &job, const void *const srcs[2], const void *const caches[2],
                void *const dsts[2], void *const stgs[2], const int64_t Ws[2], const int64_t Ps[2],
                const void *const scales[2], void *const sdsts[2], const int64_t SWs[2],
                int compress, bool &vec);

namespace {

using tdev::Table;
using tdev::TableSmem;

struct StepArgs {
  const void *ids;
  int ids_bytes;
  int64_t K, E;
  Table a, b;
  int32_t *map32;
  int32_t *map_host;  // optional copy of expert_map in device-mapped host memory
  int64_t *a_slot, *a_todo, *b_slot, *b_todo;
  gdev::CopyJob ram, ssd;  // the two copy passes
  int copy_ctas;
  int fetch;
  gdev::Fetch f;
  uint32_t *scratch;  // [0] tables done, [1] ssd done, [2] CTAs finished, [3] errors
  uint32_t *errors_out;  // optional: receives the error count when a wait gives up
  int64_t table_wait_ns, ssd_wait_ns;
};

__device__ __forceinline__ uint32_t load_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0 waits (bounded) until *flag >= target; true on every thread if it
// did.  A wait that gives up adds one to *errors and, if errors_out is set,
// stores the new count there at system scope (it may be mapped host memory
// that the host polls); concurrent give-ups may store their counts out of
// order, so errors_out can lag *errors but moves whenever a wait gives up.
__device__ bool wait_flag(const uint32_t *flag, uint32_t target, int64_t limit_ns,
                          uint32_t *errors, uint32_t *errors_out) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_ns();
    uint32_t v;
    while ((v = load_acquire_gpu(flag)) < target) {
      if (global_ns() - t0 > static_cast<uint64_t>(limit_ns)) break;
      __nanosleep(128);
    }
    s_ok = v >= target;
    if (!s_ok) {
      const uint32_t n = atomicAdd(errors, 1u) + 1u;
      if (errors_out)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(errors_out), "r"(n) : "memory");
    }
    __threadfence();
  }
  __syncthreads();
  return s_ok != 0;
}

// Publish this CTA's global writes, then raise a flag (thread 0).
__device__ void raise_flag(uint32_t *flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(flag, 1u);
  }
}

template <bool VEC>
__global__ void __launch_bounds__(gdev::kThreads) step_kernel(const __grid_constant__ StepArgs p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ gdev::CopySmem csm;
  const int role = blockIdx.x;
  uint32_t *flags = p.scratch;
  if (role < 2) {
    const int64_t S = p.a.slots > p.b.slots ? p.a.slots : p.b.slots;
    TableSmem sm = tdev::carve(smem, p.E, S);
    const bool vram = role == 0;
    const tdev::Table t = vram ? p.a : p.b;
    tdev::need_and_table(sm, t, p.ids, p.ids_bytes, p.K, p.E);
    tdev::acquire_table(sm, t, p.E, p.K, vram ? p.map32 : nullptr, nullptr,
                        vram ? p.a_slot : p.b_slot, vram ? p.a_todo : p.b_todo, true, true);
    raise_flag(&flags[0]);
    // The host copy of expert_map: written through the host link by the VRAM
    // table's CTA after the copies are released (acquire_table ended with a
    // barrier, so the map is complete).
    if (vram && p.map_host)
      for (int64_t e = threadIdx.x; e < p.E; e += blockDim.x) p.map_host[e] = p.map32[e];
  } else if (p.fetch && role == static_cast<int>(gridDim.x) - 1) {
    if (wait_flag(&flags[0], 2, p.table_wait_ns, &flags[3], p.errors_out)) {
      gdev::fetch_publish(p.f);
      __syncthreads();
      gdev::fetch_wait(p.f);
    }
    raise_flag(&flags[1]);
  } else {
    const int cta = role - 2;
    if (wait_flag(&flags[0], 2, p.table_wait_ns, &flags[3], p.errors_out)) {
      gdev::copy_rows<VEC>(p.ram, cta, p.copy_ctas, csm);
      if (p.fetch && wait_flag(&flags[1], 1, p.ssd_wait_ns, &flags[3], p.errors_out)) {
        __syncthreads();
        gdev::copy_rows<VEC>(p.ssd, cta, p.copy_ctas, csm);
      }
    }
  }
  // The last CTA to finish clears the flags for the next launch.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&flags[2], 1u) == gridDim.x - 1) {
      flags[0] = 0;
      flags[1] = 0;
      flags[2] = 0;
      __threadfence();
    }
  }
}

// Limits of the flag waits (xp_set_step_wait_ns); negative = the defaults.
std::atomic<int64_t> g_table_wait_ns{-1}, g_ssd_wait_ns{-1};
constexpr int64_t kDefaultTableWaitNs = 2'000'000'000;

// Most step CTAs that fit on the current device at once, for one kernel and
// dynamic shared memory size (cached: the occupancy query costs microseconds).
int resident_ctas(const void *fn, size_t smem, int *out) {
  struct Entry {
    int dev;
    const void *fn;
    size_t smem;
    int ctas;
  };
  static std::mutex mu;
  static Entry cache[32];
  static int used = 0;
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return static_cast<int>(err);
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].dev == dev && cache[i].fn == fn && cache[i].smem == smem) {
      *out = cache[i].ctas;
      return XP_OK;
    }
  int per_sm = 0, sms = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, gdev::kThreads, smem);
  if (err != cudaSuccess) return static_cast<int>(err);
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return static_cast<int>(err);
  *out = per_sm * sms;
  cache[used % 32] = Entry{dev, fn, smem, *out};
  used = used < 32 ? used + 1 : 32;
  return XP_OK;
}

}  // namespace
}  // namespace xp

using namespace xp;

extern "C" int xp_set_step_wait_ns(int64_t table_ns, int64_t ssd_ns) {
  if (table_ns > XP_MAX_RETRY_NS || ssd_ns > XP_MAX_RETRY_NS) return XP_EINVAL;
  g_table_wait_ns.store(table_ns < 0 ? -1 : table_ns);
  g_ssd_wait_ns.store(ssd_ns < 0 ? -1 : ssd_ns);
  return XP_OK;
}

extern "C" int xp_decode_step(
    const void *topk_ids, int ids_bytes, int64_t K, int64_t E,
    int64_t *a_slot_of, int64_t *a_expert_in, int64_t *a_last_used, int64_t *a_counters,
    int64_t a_slots, int32_t *expert_map, int32_t *expert_map_host, int64_t *a_slot,
    int64_t *a_todo,
    int64_t *b_slot_of, int64_t *b_expert_in, int64_t *b_last_used, int64_t *b_counters,
    int64_t b_slots, int64_t *b_slot, int64_t *b_todo,
    const int64_t *no_cache, int64_t base,
    const void *src0, void *dst0, void *stg0, int64_t W0, int64_t P0,
    const void *src1, void *dst1, void *stg1, int64_t W1, int64_t P1,
    const void *scale0, void *sdst0, int64_t SW0, const void *scale1, void *sdst1, int64_t SW1,
    int compress, int64_t chunk, int ctas, int64_t layer, int64_t *seq, int64_t *req,
    const int64_t *done, int64_t block, int64_t ring, int64_t retry_ns, int64_t giveup,
    uint32_t *scratch, uint32_t *errors_out, void *stream) {
  StepArgs p{};
  p.ids = topk_ids;
  p.ids_bytes = ids_bytes;
  p.K = K;
  p.E = E;
  p.a = Table{a_slot_of, a_expert_in, a_last_used, a_counters, a_slots};
  p.b = Table{b_slot_of, b_expert_in, b_last_used, b_counters, b_slots};
  p.map32 = expert_map;
  p.map_host = expert_map_host;
  p.a_slot = a_slot;
  p.a_todo = a_todo;
  p.b_slot = b_slot;
  p.b_todo = b_todo;
  if ((ids_bytes != 4 && ids_bytes != 8) || K < 0 || (K > 0 && !topk_ids) || E < 1 ||
      E > XP_MAX_EXPERTS || !expert_map || !a_slot || !a_todo || !b_slot || !b_todo ||
      !no_cache || !scratch || !aligned(scratch, 16))
    return XP_EINVAL;
  for (const Table *t : {&p.a, &p.b})
    if (!t->slot_of || !t->expert_in || !t->last_used || !t->counters || t->slots < 1 ||
        t->slots > XP_MAX_SLOTS || K > t->slots)
      return XP_EINVAL;
  if (K > gdev::kMaxK || ctas < 0 || ctas > XP_MAX_COPY_CTAS) return XP_EINVAL;
  const void *srcs[2] = {src0, src1}, *caches[2] = {dst0, dst1};
  void *dsts[2] = {dst0, dst1}, *stgs[2] = {stg0, stg1};
  const void *scales[2] = {scale0, scale1};
  void *sdsts[2] = {sdst0, sdst1};
  const int64_t Ws[2] = {W0, W1}, Ps[2] = {P0, P1}, SWs[2] = {SW0, SW1};
  bool vec;
  if (!fill_names(p.ram, srcs, caches, dsts, stgs, Ws, Ps, scales, sdsts, SWs, compress, vec))
    return XP_EINVAL;
  // Compressed rows with a known record layout: copy only each record's used words.
  if (chunk < 0) return XP_EINVAL;
  if (compress && chunk > 0) {
    if (chunk % 8) return XP_EINVAL;
    for (int i = 0; i < 2; ++i) {
      const int64_t N = 4 * Ws[i];  // raw bytes of a row
      if (N <= 0 || N % (32 * chunk)) return XP_EINVAL;
      p.ram.groups[i] = N / (32 * chunk);
    }
  }
  p.fetch = req != nullptr;
  if (p.fetch && (!seq || !done || block < 1 || ring < 1 || K > block || retry_ns < 0 ||
                  retry_ns > XP_MAX_RETRY_NS || giveup < 0 || giveup > XP_MAX_GIVEUP))
    return XP_EINVAL;
  // Pass 1: the VRAM misses that are in RAM (the SSD misses are skipped).
  p.ram.todo = a_todo;
  p.ram.K = K;
  p.ram.dst_row = a_slot;
  p.ram.cache_row = no_cache;
  p.ram.src_row = b_slot;
  p.ram.base = base;
  p.ram.skip = p.fetch ? b_todo : nullptr;
  p.ram.stage_of = nullptr;
  // Pass 2: the rows the host read (RAM misses are VRAM misses too: the RAM
  // tier holds every VRAM-tier expert), staged at their VRAM miss position.
  p.ssd = p.ram;
  p.ssd.todo = b_todo;
  p.ssd.skip = nullptr;
  p.ssd.stage_of = a_todo;
  p.copy_ctas = ctas > 0 ? ctas : 16;
  if (p.fetch)
    p.f = gdev::Fetch{b_todo, K, b_slot, base, layer, seq, seq, req, done, block, ring,
                      retry_ns, giveup};
  p.scratch = scratch;
  p.errors_out = errors_out;
  const int64_t tw = g_table_wait_ns.load(), sw = g_ssd_wait_ns.load();
  p.table_wait_ns = tw >= 0 ? tw : kDefaultTableWaitNs;
  // By default the copy CTAs outwait the fetch CTA's own bound on its SSD wait.
  p.ssd_wait_ns = sw >= 0 ? sw : (giveup + 2) * retry_ns + kDefaultTableWaitNs;
  const int64_t S = a_slots > b_slots ? a_slots : b_slots;
  const size_t smem = tdev::table_smem_bytes(E, S);
  const unsigned grid = static_cast<unsigned>(2 + p.copy_ctas + (p.fetch ? 1 : 0));
  cudaStream_t s = as_stream(stream);
  const void *fn = vec ? (const void *)step_kernel<true> : (const void *)step_kernel<false>;
  if (smem > 48 * 1024) {
    cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return static_cast<int>(err);
  }
  // The copy CTAs wait for CTAs 0/1 and the fetch CTA: all must fit at once.
  int fit = 0;
  const int orc = resident_ctas(fn, smem, &fit);
  if (orc != XP_OK) return orc;
  if (static_cast<int64_t>(grid) > fit) return XP_ERANGE;
  if (vec)
    step_kernel<true><<<grid, gdev::kThreads, smem, s>>>(p);
  else
    step_kernel<false><<<grid, gdev::kThreads, smem, s>>>(p);
  return launch_status();
}
