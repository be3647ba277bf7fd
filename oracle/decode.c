/* CPU oracle: sequential decoder of the fp8-exponent Huffman records, and a
 * threaded row copy.  TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py (its CPU baseline legs and
 * its --impl reference arm) load this library, and only as the checker or as
 * the timed CPU baseline.  The product path never links it.
 *
 * oracle_decode_row restates the sequential decoder of monochromegane/
 * vllm-expert-pager tests/test_codec.py:49-79, which walks the record format of
 * src/vllm_expert_pager/codec.py:22-26 one lane at a time with the refill rule
 * of codec.py:223-245 (one 32-bit word whenever fewer than LIMIT=9 bits remain,
 * lanes in lane order for the same symbol index).  Parity is pinned by
 * tests/test_oracle_codec.py: it decodes records made by the reference's own
 * encoder back to the raw bytes.
 *
 * oracle_copy_rows is a plain multi-threaded memcpy of whole rows: the CPU
 * stand-in for the reference's gather (src/vllm_expert_pager/gather.py:51-83),
 * which only moves bytes.
 */
#include <pthread.h>
#include <stdint.h>
#include <string.h>

#define LANES 32
#define LIMIT 9

static uint32_t rd32(const uint8_t *p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}

/* Decode group g of one record.  Returns 0, or -1 if the group reads outside
 * the record or past its own words. */
static int decode_group(const uint8_t *rec, int64_t rec_bytes, const uint8_t *lut,
                        int64_t n, int64_t chunk, int64_t g, uint8_t *out) {
  int64_t G = n / (chunk * LANES);
  int64_t nib_off = 4 * (G + 1), huff_off = nib_off + n / 2;
  int64_t rp = (int32_t)rd32(rec + 4 * g);
  int64_t end = (int32_t)rd32(rec + 4 * (g + 1));
  uint64_t buf[LANES];
  int level[LANES];
  for (int l = 0; l < LANES; l++) buf[l] = 0, level[l] = 0;
  for (int64_t i = 0; i < chunk; i++) {
    int64_t m = i / 8, k = i % 8;
    for (int l = 0; l < LANES; l++) {
      if (level[l] < LIMIT) {
        int64_t off = huff_off + 4 * rp;
        if (rp < 0 || off + 4 > rec_bytes) return -1;
        buf[l] |= (uint64_t)rd32(rec + off) << level[l];
        level[l] += 32;
        rp++;
      }
      uint8_t ent = lut[buf[l] & 511];
      buf[l] >>= (ent & 15);
      level[l] -= (ent & 15);
      uint32_t nib = rd32(rec + nib_off + 4 * ((g * (chunk / 8) + m) * LANES + l));
      uint32_t s = (nib >> (4 * k)) & 15;
      out[(g * LANES + l) * chunk + i] =
          (uint8_t)(((s & 8) << 4) | ((uint32_t)(ent >> 4) << 3) | (s & 7));
    }
  }
  return rp <= end ? 0 : -1;
}

int oracle_decode_row(const uint8_t *rec, int64_t rec_bytes, const uint8_t *lut,
                      int64_t n, int64_t chunk, uint8_t *out) {
  if (chunk <= 0 || chunk % 8 || n % (chunk * LANES)) return -2;
  int64_t G = n / (chunk * LANES);
  if (4 * (G + 1) + n / 2 > rec_bytes) return -2;
  for (int64_t g = 0; g < G; g++)
    if (decode_group(rec, rec_bytes, lut, n, chunk, g, out)) return -1;
  return 0;
}

/* ---- threaded helpers ---- */

typedef struct {
  const uint8_t *recs;
  int64_t pitch;
  const uint8_t *luts;
  int64_t rows, n, chunk;
  uint8_t *out;
  int64_t next; /* next (row, group) item, taken atomically */
  int err;
} decode_job;

static void *decode_worker(void *arg) {
  decode_job *j = (decode_job *)arg;
  int64_t G = j->n / (j->chunk * LANES);
  for (;;) {
    int64_t it = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
    if (it >= j->rows * G) return NULL;
    int64_t r = it / G, g = it % G;
    if (decode_group(j->recs + r * j->pitch, j->pitch, j->luts + r * 512, j->n, j->chunk,
                     g, j->out + r * j->n))
      __atomic_store_n(&j->err, 1, __ATOMIC_RELAXED);
  }
}

/* Decode `rows` records (pitch bytes apart, LUTs 512 B apart) into rows of n
 * bytes, on `threads` threads. */
int oracle_decode_rows(const uint8_t *recs, int64_t pitch, const uint8_t *luts, int64_t rows,
                       int64_t n, int64_t chunk, uint8_t *out, int threads) {
  if (chunk <= 0 || chunk % 8 || n % (chunk * LANES)) return -2;
  if (4 * (n / (chunk * LANES) + 1) + n / 2 > pitch) return -2;
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  decode_job j = {recs, pitch, luts, rows, n, chunk, out, 0, 0};
  pthread_t tid[256];
  for (int t = 1; t < threads; t++) pthread_create(&tid[t], NULL, decode_worker, &j);
  decode_worker(&j);
  for (int t = 1; t < threads; t++) pthread_join(tid[t], NULL);
  return j.err ? -1 : 0;
}

typedef struct {
  const uint8_t *src;
  int64_t src_pitch;
  const int64_t *src_rows;
  uint8_t *dst;
  int64_t dst_pitch;
  const int64_t *dst_rows;
  int64_t rows, row_bytes, piece;
  int64_t next;
} copy_job;

static void *copy_worker(void *arg) {
  copy_job *j = (copy_job *)arg;
  int64_t pieces = (j->row_bytes + j->piece - 1) / j->piece;
  for (;;) {
    int64_t it = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
    if (it >= j->rows * pieces) return NULL;
    int64_t r = it / pieces, p = it % pieces;
    int64_t off = p * j->piece;
    int64_t len = j->row_bytes - off < j->piece ? j->row_bytes - off : j->piece;
    memcpy(j->dst + j->dst_rows[r] * j->dst_pitch + off,
           j->src + j->src_rows[r] * j->src_pitch + off, (size_t)len);
  }
}

/* Copy rows src_rows[i] -> dst_rows[i] (row_bytes each) on `threads` threads,
 * in pieces of 256 KiB. */
int oracle_copy_rows(const uint8_t *src, int64_t src_pitch, const int64_t *src_rows,
                     uint8_t *dst, int64_t dst_pitch, const int64_t *dst_rows, int64_t rows,
                     int64_t row_bytes, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  copy_job j = {src, src_pitch, src_rows, dst, dst_pitch, dst_rows, rows, row_bytes,
                256 << 10, 0};
  pthread_t tid[256];
  for (int t = 1; t < threads; t++) pthread_create(&tid[t], NULL, copy_worker, &j);
  copy_worker(&j);
  for (int t = 1; t < threads; t++) pthread_join(tid[t], NULL);
  return 0;
}
