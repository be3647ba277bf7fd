/* xpager: C ABI of the B200-native expert-paging hot path (libxpager.so).
 *
 * Each entry point replaces one operation of monochromegane/vllm-expert-pager;
 * the comment above it cites the reference interface (file:line, paths inside
 * that project) whose arguments and semantics it keeps.  Conventions:
 *
 *  - Device functions take device pointers (or UVA pointers to pinned host
 *    memory where stated), element counts, and a cudaStream_t passed as void*
 *    (NULL = the legacy default stream).  They enqueue kernels and return at
 *    once: no host synchronisation, no device allocation, so every call can be
 *    captured in a CUDA graph.
 *  - Index arrays are int64; -1 marks an empty entry.  Expert ids may be int32
 *    or int64 (ids_bytes = 4 or 8); ids < 0 or >= E are ignored.
 *  - Return value: XP_OK, a negative XP_E* code for a bad argument (nothing was
 *    launched), or a positive cudaError_t from the launch.
 *  - A table is five device arrays: slot_of[E] (expert -> slot, -1 = not
 *    cached), expert_in[S] (slot -> expert, -1 = free), last_used[S] (step of
 *    last use, 0 = free) and counters[3] = {step, hits, misses}; the step
 *    starts at 1.  The reference keeps a trailing sink element on each array
 *    (table.py:22-26); callers may allocate it, the kernels never touch it.
 */
#ifndef XPAGER_H
#define XPAGER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XP_OK 0
#define XP_EINVAL (-22)   /* bad size, null pointer or misalignment */
#define XP_ERANGE (-34)   /* a size above the kernel's limits */
#define XP_EPITCH (-75)   /* xp_encode_row: the record does not fit the pitch */

/* Limits of the table kernels: E <= XP_MAX_EXPERTS, S <= XP_MAX_SLOTS. */
#define XP_MAX_EXPERTS 4096
#define XP_MAX_SLOTS 2048
/* Limits of the gather / fetch arguments (larger values are XP_EINVAL): copying
 * CTAs (ctas), the re-publish interval of an SSD wait (retry_ns, at most one
 * hour) and the number of re-publishes before it gives up (giveup). */
#define XP_MAX_COPY_CTAS 1024
#define XP_MAX_RETRY_NS 3600000000000LL
#define XP_MAX_GIVEUP (1 << 20)

/* Library version, and a static description of a status code. */
int xp_version(void);
const char *xp_status_string(int status);

/* ---- slot table (subsystem 1) ---- */

/* Replaces AcquirePair.__call__ / _acquire_pair_kernel (acquire.py:103-185):
 * ExpertTable.acquire (table.py:75-128) on the VRAM table a and the RAM table
 * b in one launch (one CTA per table).  Writes expert_map[E] (int32, slot of a
 * needed expert, -1 otherwise), a_slot[E] / b_slot[E] (every expert's slot
 * after the update, -1 if not cached; table.py:118 reads the updated slot_of)
 * and the miss lists a_todo[K] / b_todo[K] (missed experts in ascending id
 * order, -1 padded).  Requires K <= a_slots <= b_slots' tables' sizes as in
 * the reference (K <= S). */
int xp_acquire_pair(const void *topk_ids, int ids_bytes, int64_t K, int64_t E,
                    int64_t *a_slot_of, int64_t *a_expert_in, int64_t *a_last_used,
                    int64_t *a_counters, int64_t a_slots, int32_t *expert_map,
                    int64_t *a_slot, int64_t *a_todo,
                    int64_t *b_slot_of, int64_t *b_expert_in, int64_t *b_last_used,
                    int64_t *b_counters, int64_t b_slots, int64_t *b_slot, int64_t *b_todo,
                    void *stream);

/* Replaces ExpertTable.acquire (table.py:75-128) on one table.  expert_map
 * (int64[E]), slot[E] and todo[K] may each be NULL to skip that output.
 * Requires K <= slots. */
int xp_acquire(const void *topk_ids, int ids_bytes, int64_t K, int64_t E, int64_t *slot_of,
               int64_t *expert_in, int64_t *last_used, int64_t *counters, int64_t slots,
               int64_t *expert_map, int64_t *slot, int64_t *todo, void *stream);

/* Replaces ExpertTable.need_mask (table.py:63-71): need[e] = 1 if e occurs in
 * the ids, else 0 (uint8[E]). */
int xp_need_mask(const void *ids, int ids_bytes, int64_t K, int64_t E, uint8_t *need,
                 void *stream);

/* Replaces ExpertTable.seed (table.py:140-171) on the RAM table (R slots):
 * acquire the R-S most referenced experts of ids (if R > S), then the experts
 * of the VRAM table's expert_in[S] that are in the RAM table or in need[E];
 * hits/misses are left unchanged.  Ties among equal counts go to the lower
 * expert id (the reference's torch.topk order is implementation-defined).  If
 * top_in is not NULL it gives the max(R-S,1) experts to use instead (replays a
 * recorded choice).  If top_out is not NULL the list used is written there. */
int xp_seed(const void *ids, int ids_bytes, int64_t K, int64_t E, int64_t *slot_of,
            int64_t *expert_in, int64_t *last_used, int64_t *counters, int64_t R,
            const int64_t *vram_expert_in, int64_t S, const uint8_t *need,
            const int64_t *top_in, int64_t *top_out, void *stream);

/* Replaces ExpertTable.plan_chunks (table.py:173-247).  slot_of is the RAM
 * table after acquire/seed, before[E] its copy from before, cached_row[E] the
 * VRAM table's slot_of.  N = ceil(E/W)+1 chunks.  Outputs: dst_row[E],
 * src_row[E], maps[N*E] (row-major [N][E]), todo/ssd/late[N*W]. */
int xp_plan_chunks(int64_t E, const int64_t *slot_of, const int64_t *before,
                   const uint8_t *need, const int64_t *cached_row, int64_t W, int64_t ram_base,
                   int64_t working_base, int64_t *dst_row, int64_t *src_row, int64_t *maps,
                   int64_t *todo, int64_t *ssd, int64_t *late, void *stream);

/* The planning of one working-path step in one launch: replaces the sequence
 * need_mask -> slot_of[:E].clone() -> acquire (K <= R) or seed -> plan_chunks
 * of _expert_pager_forward_working (experts.py:500-511) on the RAM table
 * (R slots), given the VRAM table's expert_in[S] and slot_of (cached_row[E]).
 * Writes need[E] (uint8) and before[E] (slot_of before the update) and the
 * outputs of xp_plan_chunks; top_in / top_out as in xp_seed.  Results equal
 * the separate calls'.  No counterpart in the reference (it issues those
 * steps as separate torch operations). */
int xp_plan_working(const void *ids, int ids_bytes, int64_t K, int64_t E, int64_t *slot_of,
                    int64_t *expert_in, int64_t *last_used, int64_t *counters, int64_t R,
                    const int64_t *vram_expert_in, const int64_t *cached_row, int64_t S,
                    int64_t W, int64_t ram_base, int64_t working_base, const int64_t *top_in,
                    int64_t *top_out, uint8_t *need, int64_t *before, int64_t *dst_row,
                    int64_t *src_row, int64_t *maps, int64_t *todo, int64_t *ssd,
                    int64_t *late, void *stream);

/* ---- gather (subsystem 2) and the SSD request ring ---- */

/* Replaces gather_rows / _gather_rows_kernel (gather.py:149-194,328-393).
 * Rows are counted in 32-bit words like the reference's as_rows views.  For
 * each todo[j] = e >= 0 (and, if skip is not NULL, e not in skip[0:K]):
 *   cache_row[e] >= 0: cache_n[cache_row[e]] (W_n words) -> dst_n[dst_row[e]];
 *   else compress:     src_n[src_row[e]+base] (P_n words) -> stg_n[j];
 *   else:              src_n[src_row[e]+base] (P_n == W_n) -> dst_n[dst_row[e]];
 * and always scale_n[e] (SW_n words) -> sdst_n[dst_row[e]], for names n = 0, 1.
 * src_n may be pinned host memory (read over the host link by the SMs).
 * chunk (compressed rows only; not in the reference): the records' values per
 * lane; when > 0 (and at most 64 entries are copied from the RAM tier) only each
 * record's used words -- header, nibbles, Huffman words, read from its header --
 * cross the host link, as in xp_decode_step; 0 copies whole P_n-word records.
 * ctas: copying CTAs (0 = default).  If req is not NULL, one more CTA runs
 * xp_fetch on skip (the decode path's fused publish + wait, gather.py:170-185);
 * its arguments are those of xp_fetch. */
int xp_gather_rows(const int64_t *todo, int64_t K, const int64_t *dst_row,
                   const int64_t *cache_row, const int64_t *src_row, int64_t base,
                   const void *src0, const void *cache0, void *dst0, void *stg0, int64_t W0,
                   int64_t P0,
                   const void *src1, const void *cache1, void *dst1, void *stg1, int64_t W1,
                   int64_t P1,
                   const void *scale0, void *sdst0, int64_t SW0,
                   const void *scale1, void *sdst1, int64_t SW1,
                   const int64_t *skip, int compress, int64_t chunk, int ctas,
                   int64_t layer, int64_t *seq, int64_t *req, const int64_t *done,
                   int64_t block, int64_t ring, int64_t retry_ns, int64_t giveup,
                   void *stream);

/* Replaces fetch_publish_rows / _fetch_publish (gather.py:197-234,410-431):
 * if todo[0:K] has an entry >= 0, take seq = ++*seq, write *ticket = seq and
 * publish request slot seq % ring of req (pinned, UVA): [seq, layer,
 * expert[block], row[block]] with row = row_of[e] + base, -1 padded, seq
 * stored last with release semantics at system scope.  req[0] counts
 * re-publishes and req[1] give-ups.  Otherwise nothing is written. */
int xp_fetch_publish(const int64_t *todo, int64_t K, const int64_t *row_of, int64_t base,
                     int64_t layer, int64_t *seq, int64_t *ticket, int64_t *req, int64_t block,
                     int64_t ring, void *stream);

/* Replaces fetch_wait_rows / _fetch_wait (gather.py:237-277,434-439): if
 * todo[0:K] has an entry >= 0, wait until *done >= *ticket (done is pinned and
 * written by the host server).  Every retry_ns nanoseconds of waiting the
 * request is published again and req[0] incremented; after giveup such
 * re-publishes the wait ends and req[1] is incremented (the reference uses
 * 2^18 spins and 8 tries).  The wait never blocks longer than about
 * (giveup+1) * retry_ns. */
int xp_fetch_wait(const int64_t *todo, int64_t K, const int64_t *ticket, int64_t *req,
                  const int64_t *done, int64_t block, int64_t ring, int64_t retry_ns,
                  int64_t giveup, void *stream);

/* Replaces fetch_rows / _fetch_kernel (gather.py:280-296,396-407): publish and
 * wait in one launch; the ticket is *seq itself. */
int xp_fetch(const int64_t *todo, int64_t K, const int64_t *row_of, int64_t base, int64_t layer,
             int64_t *seq, int64_t *req, const int64_t *done, int64_t block, int64_t ring,
             int64_t retry_ns, int64_t giveup, void *stream);

/* Bytes of the scratch block xp_decode_step needs (zeroed once by the caller;
 * every launch leaves it zeroed again except the error counter, word 3). */
#define XP_STEP_SCRATCH_BYTES 16

/* No counterpart in the reference.  Limits, in nanoseconds, of the fused
 * step's waits on its own CTAs: table_ns for the table updates (default 2 s),
 * ssd_ns for the SSD fetch CTA (default (giveup + 2) * retry_ns + 2 s, longer
 * than the fetch CTA's own bounded wait).  A negative value restores the
 * default; values above XP_MAX_RETRY_NS are XP_EINVAL.  Process-wide, read at
 * each launch.  A wait that runs out is counted as a give-up (see
 * xp_decode_step); tests use short limits to make one run out. */
int xp_set_step_wait_ns(int64_t table_ns, int64_t ssd_ns);

/* Replaces the decode path's three launches (experts.py:406-447: AcquirePair,
 * gather_rows with fetch, gather_rows of the SSD misses) with one: CTA 0/1
 * update the VRAM table a and the RAM table b exactly as xp_acquire_pair
 * (same outputs), the copy CTAs then copy the VRAM misses from the RAM tier
 * (src_n rows b_slot[e] + base; to dst_n[a_slot[e]] raw, or to the staging row
 * of e's position in a_todo when compressed) with their scale rows, and, if
 * req is not NULL, a last CTA publishes the RAM misses (b_todo) to the host
 * server and waits as xp_fetch does, after which the copy CTAs copy those rows
 * too.  A compressed step then needs one xp_decode_rows(a_todo, a_slot,
 * no_cache, ...) without skip.  no_cache: int64[E] of -1.  scratch:
 * XP_STEP_SCRATCH_BYTES of device memory, 16-byte aligned, zeroed before the
 * first call and not shared by launches that may overlap; scratch word 3
 * (uint32) counts waits that gave up (the rows of that step are then stale).
 * errors_out (may be NULL; no counterpart in the reference): device memory or
 * device-mapped pinned host memory into which a wait that gives up stores the
 * new count, so that the host can watch for give-ups without a
 * synchronisation.  topk_ids may be pinned host memory (read through the host
 * link).  expert_map_host (may be NULL; no counterpart in the reference) is
 * device-mapped pinned host memory that receives a copy of expert_map[E] from
 * the kernel, so that a host-driven caller needs no copy-engine transfer per
 * step.  The copy CTAs wait for the others, so the launch is refused with
 * XP_ERANGE when its 2 + ctas (+1 with req) CTAs cannot all be resident on the
 * device at once.  chunk (no counterpart in the reference, which copies whole
 * records): with compress, the records' values per lane; then only each
 * record's used words (its header, nibbles and Huffman words, known from the
 * header) are copied to staging, the rest of the staging row is left as it was
 * (the decode never reads it).  0 copies whole P-word records. */
int xp_decode_step(const void *topk_ids, int ids_bytes, int64_t K, int64_t E,
                   int64_t *a_slot_of, int64_t *a_expert_in, int64_t *a_last_used,
                   int64_t *a_counters, int64_t a_slots, int32_t *expert_map,
                   int32_t *expert_map_host, int64_t *a_slot, int64_t *a_todo,
                   int64_t *b_slot_of, int64_t *b_expert_in, int64_t *b_last_used,
                   int64_t *b_counters, int64_t b_slots, int64_t *b_slot, int64_t *b_todo,
                   const int64_t *no_cache, int64_t base,
                   const void *src0, void *dst0, void *stg0, int64_t W0, int64_t P0,
                   const void *src1, void *dst1, void *stg1, int64_t W1, int64_t P1,
                   const void *scale0, void *sdst0, int64_t SW0,
                   const void *scale1, void *sdst1, int64_t SW1,
                   int compress, int64_t chunk, int ctas, int64_t layer, int64_t *seq,
                   int64_t *req, const int64_t *done, int64_t block, int64_t ring,
                   int64_t retry_ns, int64_t giveup, uint32_t *scratch, uint32_t *errors_out,
                   void *stream);

/* Size of the device array xp_decode_step_noalloc takes its scratch from. */
#define XP_NOALLOC_SCRATCH_BYTES (32u << 20)

/* No counterpart in the reference.  For callers that cannot allocate device
 * memory (an engine that reserved all free memory for its own pools, or a
 * host that only has this C ABI): xp_decode_step plus, when compressed, the
 * decode of every VRAM miss (xp_decode_rows with a_todo, a_slot, no_cache,
 * lut, chunk), with the flag block and the staging rows taken from a fixed
 * XP_NOALLOC_SCRATCH_BYTES array compiled into the library, held by every GPU
 * that loads it.  Row sizes W/P are in 32-bit words as in xp_decode_step.
 * Returns XP_ERANGE (nothing launched) if K > 2048 or if 256 + K*(P0+P1)*4
 * staging bytes do not fit the array.  The first call on a device looks the
 * array up (which may load the library's device code: make that call before
 * any stream capture) and queues a clear of its flags on `stream`; the address
 * is kept for the life of the device's primary context, so do not call this
 * again after cudaDeviceReset.  All calls on a device share the array; calls
 * that overlap on the GPU race.  errors_out (may be NULL) receives the running
 * count of the step's waits that gave up, as in xp_decode_step: the array's
 * own counter is not reachable from the host. */
int xp_decode_step_noalloc(const void *topk_ids, int ids_bytes, int64_t K, int64_t E,
                           int64_t *a_slot_of, int64_t *a_expert_in, int64_t *a_last_used,
                           int64_t *a_counters, int64_t a_slots, int32_t *expert_map,
                           int64_t *a_slot, int64_t *a_todo,
                           int64_t *b_slot_of, int64_t *b_expert_in, int64_t *b_last_used,
                           int64_t *b_counters, int64_t b_slots, int64_t *b_slot, int64_t *b_todo,
                           const int64_t *no_cache, int64_t base,
                           const void *src0, void *dst0, int64_t W0, int64_t P0,
                           const void *src1, void *dst1, int64_t W1, int64_t P1,
                           const void *scale0, void *sdst0, int64_t SW0,
                           const void *scale1, void *sdst1, int64_t SW1,
                           int compress, const uint8_t *lut, int64_t chunk, int ctas,
                           int64_t layer, int64_t *seq, int64_t *req, const int64_t *done,
                           int64_t block, int64_t ring, int64_t retry_ns, int64_t giveup,
                           uint32_t *errors_out, void *stream);

/* ---- decode (subsystem 3) ---- */

/* Replaces decode_rows / _decode_rows_kernel (codec.py:248-327).  For each
 * todo[j] = e >= 0 with cache_row[e] < 0 (and e not in skip[0:K] if skip is
 * not NULL): expand record stg_n[j] (P_n bytes per row) into dst_n[dst_row[e]]
 * (N_n bytes per row) with the LUT lut[e][n] (uint8[E][2][512]), n = 0, 1.
 * chunk: values per lane (512 in production; multiple of 8, at most 2^30; N_n
 * a multiple of 32*chunk).  stg_n and dst_n start on 16-byte boundaries and P_n
 * is a multiple of 16 (else XP_EINVAL); rows on 32-byte boundaries with chunk a
 * multiple of 32 are written with 32-byte stores.  Records are in the
 * reference's format (codec.py:22-26). */
int xp_decode_rows(const int64_t *todo, int64_t K, const int64_t *dst_row,
                   const int64_t *cache_row, const uint8_t *lut,
                   const void *stg0, int64_t P0, void *dst0, int64_t N0,
                   const void *stg1, int64_t P1, void *dst1, int64_t N1,
                   const int64_t *skip, int64_t chunk, void *stream);

/* Replaces codec.encode (codec.py:125-193), which the reference runs as torch
 * ops on the GPU while loading weights (store.py:576-599), for a batch of rows:
 * raw[rows][n] (device, 16-byte aligned) -> records[rows][pitch] (zero padded
 * past each record's used bytes) and luts[rows][512], byte-identical to the
 * reference.  used[rows] (device) receives each record's used bytes; a row with
 * used > pitch is not written (the caller checks, as codec.py:157-162 raises).
 * scratch: device memory of at least xp_encode_scratch_bytes(rows, n, chunk)
 * bytes, 256-byte aligned.  n must be a multiple of 32*chunk, chunk of 8; rows
 * <= 65535.  Five launches on `stream`, no allocation, no synchronisation. */
int64_t xp_encode_scratch_bytes(int64_t rows, int64_t n, int64_t chunk);
int xp_encode_rows(const void *raw, int64_t rows, int64_t n, int64_t pitch, int64_t chunk,
                   void *records, void *luts, int64_t *used, void *scratch,
                   int64_t scratch_bytes, void *stream);

/* ---- host side ---- */

/* Replaces codec.encode (codec.py:125-193) on the host: compress raw[n] into
 * record[pitch] (zero padded) and lut[512].  *used receives the record's used
 * bytes.  Returns XP_EPITCH if used > pitch (record unspecified), XP_EINVAL if
 * n is not a multiple of 32*chunk. */
int xp_encode_row(const uint8_t *raw, int64_t n, int64_t pitch, int64_t chunk, uint8_t *record,
                  uint8_t *lut, int64_t *used);

/* Pinned, device-mapped host memory of `bytes` bytes (4 KiB aligned) placed on
 * NUMA node `numa_node` (-1: no placement).  Replaces Store's torch pinned
 * allocation (store.py:334-348,408-421).  *dev receives the device (UVA)
 * address. */
int xp_pinned_alloc(int64_t bytes, int numa_node, void **host, void **dev);
int xp_pinned_free(void *host, int64_t bytes);
/* Device address of a pinned host pointer (vLLM's
 * get_accelerator_view_from_cpu_tensor, store.py:430-432,450-451). */
int xp_device_pointer(void *host, void **dev);

/* The SSD request server: same ABI as the reference's C server
 * (store.py:253-308, bound at store.py:312-331).  Serves ring requests in seq
 * order with `nworkers`+1 concurrent preadv's of record_bytes at offset
 * (layer*E + e)*record_bytes into pinned rows; writes *done = seq (release)
 * when a request is complete, even if a read failed. */
void *ssd_start(int fd, void *req, void *done, long ring, long block, long L, long E, long rows,
                long record_bytes, int names, void **pinned, long *pitch, int nworkers);
void ssd_stop(void *server);
void ssd_stats(void *server, long *fetches, long *reads, double *io_seconds, long *missed);
const char *ssd_error(void *server);
void ssd_test_delay(void *server, double seconds);
/* No counterpart in the reference: the NUMA node whose CPUs the server's
 * threads were bound to at ssd_start (the node holding pinned[0]'s first page,
 * found with get_mempolicy), or -1 if the kernel did not report one. */
int ssd_numa_node(void *server);
/* No counterpart in the reference: split every record read of later requests
 * into jobs of `bytes` (rounded down to whole 4 KiB pages; 0, or at least
 * record_bytes: one job per record, the reference's behaviour), read by the
 * server's threads concurrently.  A request of one or two experts then keeps
 * nworkers+1 reads in flight instead of one or two. */
void ssd_set_read_chunk(void *server, long bytes);
/* No counterpart in the reference: used[(layer*E + e)*names + i] gives the
 * bytes of name i's piece of record (layer, e) that hold data (for compressed
 * records: header, nibbles and Huffman words; 0, or at least the piece's
 * pitch: the whole piece).  Later requests read each piece only up to its last
 * data page (when every pitch is a whole number of 4 KiB pages, as Store's are;
 * else whole records), so the disk moves ~7 % fewer bytes per compressed record; the
 * rest of the RAM-tier row keeps old bytes, which the decoder never reads.
 * The array is the caller's and must outlive the server (NULL: whole records). */
void ssd_set_used_bytes(void *server, const long *used);
/* No counterpart in the reference: bytes the server has read from the file. */
long ssd_bytes_read(void *server);

#ifdef __cplusplus
}
#endif

#endif /* XPAGER_H */
