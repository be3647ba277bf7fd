// Host server of the SSD tier: serves the GPU's read requests from the paging
// file into pinned RAM-tier rows.
//
// Keeps the C ABI and protocol of monochromegane/vllm-expert-pager
// src/vllm_expert_pager/store.py:68-309 (bound by ctypes at store.py:312-331):
//  * req = [re-publishes, give-ups] + ring slots of [seq, layer, expert[B], row[B]];
//    the GPU publishes seq last with release semantics (gather.cu);
//  * requests are served in seq order; done = seq is stored with release
//    semantics once every read of the request finished, even if one failed;
//  * a read is one preadv of record_bytes at (layer*E + e)*record_bytes into
//    the row's pinned pieces (one per name), with bounds checks;
//  * while idle the server rewrites done when the GPU's re-publish counter
//    moves or after 2^25 idle spins (a lost done), counts seq gaps as missed,
//    and honours a test-only delay.
//
// Implementation: one server thread spinning on the ring (a sleep adds ~100 us
// to the round trip) and a pool of worker threads that take jobs one at a time
// under a mutex (a job is a read of hundreds of kilobytes to a few megabytes).
// All of them run on the CPUs of the NUMA node that holds the RAM tier.  A job
// is one record, or, when ssd_set_read_chunk set a chunk size, one page-aligned
// chunk of a record: a request of one or two experts then keeps every reader
// busy instead of one or two (a disk reaches its bandwidth only with several
// reads in flight).
//
// Requests are pipelined: once every job of the oldest request has been taken
// (some may still be reading), the server admits the next published request
// and queues its jobs behind, up to kPipeline requests in flight, so the
// readers do not drain between consecutive requests (the working path
// publishes chunk k+1's request before it waits for chunk k's).  done still
// advances in seq order, each value stored only after every read of that
// request and of the ones before it finished.  The reference serves one
// request at a time (store.py:231-239).
#define _GNU_SOURCE 1
#include <errno.h>
#include <pthread.h>
#include <sched.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/syscall.h>
#include <sys/uio.h>
#include <time.h>
#include <unistd.h>

#include <atomic>
#include <condition_variable>
#include <mutex>
#include <thread>
#include <vector>

#include "xpager.h"

namespace {

constexpr int kMaxNames = 4;
constexpr long kHead = 2;

double now_s() {
  timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return static_cast<double>(t.tv_sec) + 1e-9 * static_cast<double>(t.tv_nsec);
}

inline void cpu_relax(long &spins) {
  if (++spins > 200000) {
    sched_yield();
    spins = 0;
  } else {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#elif defined(__aarch64__)
    asm volatile("yield");
#endif
  }
}

int64_t load_acq(const volatile int64_t *p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
void store_rel(volatile int64_t *p, int64_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }

// NUMA node of the page at addr (get_mempolicy(2) with MPOL_F_NODE |
// MPOL_F_ADDR, spelled out to avoid libnuma), -1 if the kernel does not say.
int node_of(const void *addr) {
  constexpr unsigned long kNode = 1ul << 0, kAddr = 1ul << 1;
  int node = -1;
  const long rc = syscall(SYS_get_mempolicy, &node, nullptr, 0ul, addr, kNode | kAddr);
  return rc == 0 ? node : -1;
}

// CPUs of a NUMA node from sysfs ("0-15,32-47"); false if unreadable or empty.
bool node_cpus(int node, cpu_set_t *set) {
  char path[96];
  snprintf(path, sizeof path, "/sys/devices/system/node/node%d/cpulist", node);
  FILE *f = fopen(path, "r");
  if (!f) return false;
  char buf[4096];
  const bool got = fgets(buf, sizeof buf, f) != nullptr;
  fclose(f);
  if (!got) return false;
  CPU_ZERO(set);
  int count = 0;
  for (char *p = buf; *p && *p != '\n';) {
    char *end;
    long a = strtol(p, &end, 10);
    if (end == p) return false;
    long b = a;
    if (*end == '-') {
      p = end + 1;
      b = strtol(p, &end, 10);
      if (end == p) return false;
    }
    for (long c = a; c <= b && c < CPU_SETSIZE; ++c, ++count) CPU_SET(static_cast<int>(c), set);
    p = *end == ',' ? end + 1 : end;
  }
  return count > 0;
}

constexpr int kPipeline = 2;  // requests in flight at once

struct Server {
  int fd;
  int numa_node = -1;  // node the threads are bound to, -1 if not bound
  volatile int64_t *req, *done;
  long ring, block, slot_words, L, E, rows, record_bytes;
  int names;
  uint8_t *pinned[kMaxNames];
  long pitch[kMaxNames];

  // statistics (written by the server thread)
  std::atomic<long> fetches{0}, reads{0}, missed{0};
  std::atomic<double> io_seconds{0.0};
  char err[512];
  std::atomic<int> failing{0}, failed{0};
  std::atomic<double> test_delay{0.0};
  std::atomic<long> read_chunk{0};  // bytes per job, 0: whole records
  // Optional: the bytes of each record piece that hold data, used[(layer*E +
  // e)*names + i] (0 or more than the pitch: the whole piece); caller-owned.
  std::atomic<const long *> used{nullptr};
  std::atomic<long> bytes_read{0};

  // A job: bytes [lo, hi) of one record, read into that record's row; tag is
  // the slot of its request in the ring of kPipeline requests in flight.
  struct Job {
    long layer, expert, row, lo, hi;
    int tag;
  };
  // Jobs of the requests in flight, in admission order.  Taking a job (a copy
  // of it) happens under mu, so appending jobs cannot race with a reader.
  std::vector<Job> jobs;
  long next = 0;
  std::atomic<long> finished[kPipeline];
  std::mutex mu;
  std::condition_variable cv;
  long gen = 0;
  std::atomic<bool> stop{false};
  std::vector<std::thread> workers;
  std::thread server;

  void fail(const char *fmt, ...) {
    int expected = 0;
    if (!failing.compare_exchange_strong(expected, 1)) return;  // keep the first failure
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, sizeof err, fmt, ap);
    va_end(ap);
    failed.store(1, std::memory_order_release);
  }

  // The record is the names' pieces back to back (pitch[0] bytes of name 0,
  // then name 1, ...), each read into the row's pinned piece of that name.
  void read_one(const Job &jb) {
    const long e = jb.expert, row = jb.row, layer = jb.layer;
    if (layer < 0 || layer >= L || e < 0 || e >= E) {
      fail("expert %ld of layer %ld is out of range", e, layer);
      return;
    }
    if (row < 0 || row >= rows) {
      fail("row %ld for expert %ld of layer %ld is outside the RAM tier of %ld rows", row, e,
           layer, rows);
      return;
    }
    iovec iov[kMaxNames];
    int k = 0;
    long base = 0;
    for (int i = 0; i < names; ++i) {
      const long a = jb.lo > base ? jb.lo : base;
      const long b = jb.hi < base + pitch[i] ? jb.hi : base + pitch[i];
      if (a < b) {
        iov[k].iov_base = pinned[i] + row * pitch[i] + (a - base);
        iov[k].iov_len = static_cast<size_t>(b - a);
        ++k;
      }
      base += pitch[i];
    }
    const off_t off = static_cast<off_t>(layer * E + e) * record_bytes + jb.lo;
    ssize_t n = preadv(fd, iov, k, off);
    if (n > 0) bytes_read.fetch_add(static_cast<long>(n), std::memory_order_relaxed);
    if (n < 0)
      fail("preadv of expert %ld of layer %ld failed: %s", e, layer, strerror(errno));
    else if (n != jb.hi - jb.lo)
      fail("short read: %zd of %ld B at byte %ld of expert %ld of layer %ld", n, jb.hi - jb.lo,
           jb.lo, e, layer);
  }

  // Takes and reads one job; false if none is waiting.
  bool run_one() {
    Job jb;
    {
      std::lock_guard<std::mutex> lk(mu);
      if (next >= static_cast<long>(jobs.size())) return false;
      jb = jobs[static_cast<size_t>(next++)];
    }
    read_one(jb);
    finished[jb.tag].fetch_add(1, std::memory_order_release);
    return true;
  }

  void worker_main() {
    long seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu);
        cv.wait(lk, [&] { return gen != seen || stop.load(); });
        if (stop.load()) return;
        seen = gen;
      }
      while (run_one()) {
      }
    }
  }

  struct InFlight {
    int64_t seq;
    long experts, njobs;
    double t0;
  };

  // Queues the jobs of the request in `slot` under in-flight slot `tag` and
  // records its number of experts and jobs in f.
  void admit(volatile int64_t *slot, int tag, InFlight &f) {
    finished[tag].store(0, std::memory_order_relaxed);
    std::lock_guard<std::mutex> lk(mu);
    const long layer = static_cast<long>(slot[1]);
    // Chunks are whole pages (O_DIRECT), and only used when the record is
    // exactly the names' pieces (always, for records written by Store).
    long c = read_chunk.load(std::memory_order_relaxed) / 4096 * 4096;
    long sum = 0;
    bool paged = true;  // every piece starts on a page (O_DIRECT offsets)
    for (int i = 0; i < names; ++i) {
      sum += pitch[i];
      paged = paged && pitch[i] % 4096 == 0;
    }
    if (c <= 0 || c >= record_bytes || sum != record_bytes) c = record_bytes;
    if (next >= static_cast<long>(jobs.size())) {  // every queued job taken: start afresh
      jobs.clear();
      next = 0;
    }
    // With used lengths (records laid out as the names' pieces), each piece is
    // read only up to its last data page: the decoder never looks past a
    // record's used words.
    const long *u = sum == record_bytes && paged ? used.load(std::memory_order_acquire) : nullptr;
    long n = 0, nj = 0;
    for (long j = 0; j < block; ++j) {
      const int64_t e = slot[2 + j];
      if (e < 0) continue;
      const long row = static_cast<long>(slot[2 + block + j]);
      const bool in_range = layer >= 0 && layer < L && e >= 0 && e < E;
      long base = 0;
      for (int i = 0; i < (u && in_range ? names : 1); ++i) {
        long lo0 = 0, hi0 = record_bytes;
        if (u && in_range) {
          long len = u[(layer * E + e) * names + i];
          len = len <= 0 || len >= pitch[i] ? pitch[i] : (len + 4095) / 4096 * 4096;
          lo0 = base;
          hi0 = base + (len < pitch[i] ? len : pitch[i]);
          base += pitch[i];
        }
        for (long lo = lo0; lo < hi0; lo += c, ++nj)
          jobs.push_back(Job{layer, static_cast<long>(e), row, lo, lo + c < hi0 ? lo + c : hi0,
                             tag});
      }
      ++n;
    }
    f.experts = n;
    f.njobs = nj;
    if (nj > 1 && !workers.empty()) {  // a single job is read here without waking anyone
      ++gen;
      cv.notify_all();
    }
  }

  void server_main() {
    int64_t admitted = 0, retired = 0, retries = 0;
    InFlight fl[kPipeline];
    int head = 0, count = 0;  // ring of in-flight requests, oldest at head
    long spins = 0, idle = 0;
    for (;;) {
      if (stop.load(std::memory_order_acquire)) return;
      bool progress = false;
      // Admit the next published request while there is room and every job of
      // the requests in flight has been taken.
      if (count < kPipeline) {
        bool drained;
        {
          std::lock_guard<std::mutex> lk(mu);
          drained = next >= static_cast<long>(jobs.size());
        }
        volatile int64_t *slot = req + kHead + ((admitted + 1) % ring) * slot_words;
        const int64_t seq = drained || count == 0 ? load_acq(slot) : admitted;
        if (seq > admitted) {
          const double t0 = now_s();
          // Requests skipped over were given up by the GPU before they arrived.
          if (seq > admitted + 1) missed.fetch_add(static_cast<long>(seq - admitted - 1));
          while (test_delay.load() > 0 && now_s() - t0 < test_delay.load()) {
            if (stop.load(std::memory_order_acquire)) return;
            usleep(1000);
          }
          const int tag = (head + count) % kPipeline;
          InFlight &f = fl[tag];
          f.seq = seq;
          f.t0 = t0;
          admit(slot, tag, f);
          ++count;
          admitted = seq;
          progress = true;
        }
      }
      // Retire the oldest request once all its reads finished: done = its seq.
      while (count > 0) {
        InFlight &f = fl[head];
        if (finished[head].load(std::memory_order_acquire) < f.njobs) break;
        fetches.fetch_add(1);
        reads.fetch_add(f.experts);
        io_seconds.store(io_seconds.load() + (now_s() - f.t0));
        // Re-publishes during a long read are not lost handoffs.
        retries = load_acq(&req[0]);
        store_rel(done, f.seq);
        retired = f.seq;
        head = (head + 1) % kPipeline;
        --count;
        progress = true;
      }
      if (count > 0 && run_one()) progress = true;
      if (progress) {
        spins = 0;
        idle = 0;
        continue;
      }
      if (count == 0) {
        // Idle.  The GPU may not have seen done: rewrite it when the re-publish
        // count moves, or after a long idle period (store.py:200-207).
        int64_t r = load_acq(&req[0]);
        if (r != retries || ++idle > (1L << 25)) {
          retries = r;
          idle = 0;
          store_rel(done, retired);
        }
      }
      cpu_relax(spins);
    }
  }
};

}  // namespace

extern "C" void *ssd_start(int fd, void *req, void *done, long ring, long block, long L, long E,
                           long rows, long record_bytes, int names, void **pinned, long *pitch,
                           int nworkers) {
  if (names < 1 || names > kMaxNames || !req || !done || ring < 1 || block < 1 || nworkers < 0)
    return nullptr;
  Server *s = new (std::nothrow) Server();
  if (!s) return nullptr;
  s->fd = fd;
  s->req = static_cast<volatile int64_t *>(req);
  s->done = static_cast<volatile int64_t *>(done);
  s->ring = ring;
  s->block = block;
  s->slot_words = 2 + 2 * block;
  s->L = L;
  s->E = E;
  s->rows = rows;
  s->record_bytes = record_bytes;
  s->names = names;
  for (int i = 0; i < names; ++i) {
    s->pinned[i] = static_cast<uint8_t *>(pinned[i]);
    s->pitch[i] = pitch[i];
  }
  s->err[0] = 0;
  for (auto &f : s->finished) f.store(0);
  for (int i = 0; i < nworkers; ++i) s->workers.emplace_back([s] { s->worker_main(); });
  s->server = std::thread([s] { s->server_main(); });
  // The reads land in the RAM tier: run the server and its workers on the CPUs
  // of the NUMA node that holds it (the GPU's node, where the tier is placed).
  const int node = node_of(s->pinned[0]);
  cpu_set_t set;
  if (node >= 0 && node_cpus(node, &set)) {
    bool ok = pthread_setaffinity_np(s->server.native_handle(), sizeof set, &set) == 0;
    for (auto &t : s->workers)
      ok = pthread_setaffinity_np(t.native_handle(), sizeof set, &set) == 0 && ok;
    if (ok) s->numa_node = node;
  }
  return s;
}

extern "C" int ssd_numa_node(void *server) {
  const Server *s = static_cast<const Server *>(server);
  return s ? s->numa_node : -1;
}

extern "C" void ssd_stop(void *server) {
  Server *s = static_cast<Server *>(server);
  if (!s) return;
  {
    std::lock_guard<std::mutex> lk(s->mu);
    s->stop.store(true);
    s->cv.notify_all();
  }
  s->server.join();
  for (auto &t : s->workers) t.join();
  delete s;
}

extern "C" void ssd_stats(void *server, long *fetches, long *reads, double *io_seconds,
                          long *missed) {
  Server *s = static_cast<Server *>(server);
  *fetches = s->fetches.load();
  *reads = s->reads.load();
  *io_seconds = s->io_seconds.load();
  *missed = s->missed.load();
}

extern "C" const char *ssd_error(void *server) {
  Server *s = static_cast<Server *>(server);
  return s->failed.load(std::memory_order_acquire) ? s->err : nullptr;
}

extern "C" void ssd_set_read_chunk(void *server, long bytes) {
  if (!server) return;
  static_cast<Server *>(server)->read_chunk.store(bytes < 0 ? 0 : bytes, std::memory_order_relaxed);
}

extern "C" void ssd_set_used_bytes(void *server, const long *used) {
  if (!server) return;
  static_cast<Server *>(server)->used.store(used, std::memory_order_release);
}

extern "C" long ssd_bytes_read(void *server) {
  if (!server) return 0;
  return static_cast<Server *>(server)->bytes_read.load(std::memory_order_relaxed);
}

extern "C" void ssd_test_delay(void *server, double seconds) {
  static_cast<Server *>(server)->test_delay.store(seconds);
}
