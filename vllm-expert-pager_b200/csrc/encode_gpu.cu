// Batched GPU encoder of the fp8-exponent Huffman records (load time).
//
// Produces records and LUTs byte-identical to monochromegane/vllm-expert-pager
// src/vllm_expert_pager/codec.py:125-193 (the record format of codec.py:22-26),
// which the reference runs as torch ops on the GPU when it loads weights
// (store.py:576-599): the length-limited Huffman construction of codec.py:61-87
// with the heap's tie order, the canonical bit-reversed codes of codec.py:90-114,
// and the Huffman words of each group in refill order (codec.py:150-181).
//
// A scratch clear and five launches per batch of rows, all on the caller's
// stream, no allocation:
//   1. hist   exponent histogram per row (packed 8-bit counters per thread);
//   2. code   code lengths + canonical codes + LUT, one warp per row;
//   3. count  Huffman words per group (sum of the lanes' refill counts);
//   4. scan   group starts gstart[G+1], record size, header, zeroed tail;
//   5. emit   one warp per group: sign/mantissa nibbles, and the words.  The warp
//             replays the decoder's refill protocol from the code lengths alone
//             (a lane refills before symbol i when 32*refills - before[i] < LIMIT;
//             lanes refilling at the same i take consecutive words in lane order),
//             so each lane learns the slot of its k-th word before the word's
//             first bit is produced and stores it when its 32 bits are complete.
#include "common.cuh"

#include <cub/block/block_scan.cuh>

namespace xp {
namespace {

constexpr int kLimit = 9;
constexpr int kLutBytes = 512;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kHistThreads = 256;
constexpr int kHistBlocksPerRow = 32;
constexpr int kWarpsPerBlock = 4;
constexpr int kScanThreads = 256;

// Per-row scratch: hist[16] u32 | tab[16] u32 (code | len << 16) | lens u64 |
// pad | gw[G] i32 | gstart[G+1] i32, rounded up to 256 bytes.
__host__ __device__ inline int64_t row_scratch_bytes(int64_t G) {
  return (64 + 64 + 8 + 8 + 4 * (2 * G + 1) + 255) / 256 * 256;
}

struct RowScratch {
  uint32_t *hist, *tab;
  unsigned long long *lens;
  int32_t *gw, *gstart;
};

__device__ inline RowScratch row_scratch(unsigned char *base, int64_t row, int64_t G) {
  unsigned char *p = base + row * row_scratch_bytes(G);
  RowScratch r;
  r.hist = reinterpret_cast<uint32_t *>(p);
  r.tab = reinterpret_cast<uint32_t *>(p + 64);
  r.lens = reinterpret_cast<unsigned long long *>(p + 128);
  r.gw = reinterpret_cast<int32_t *>(p + 144);
  r.gstart = r.gw + G;
  return r;
}

struct EncArgs {
  const uint8_t *raw;  // [rows][n]
  int64_t rows, n, pitch, chunk, G;
  uint8_t *records;  // [rows][pitch]
  uint8_t *luts;     // [rows][512]
  int64_t *used;     // [rows]
  unsigned char *scratch;
};

// 1. Histogram of the exponent field (bits 3..6) of every byte.  Each thread
// keeps its 16 counts as 8-bit fields of two 64-bit registers and flushes
// them to shared memory before a field could reach 256.
__global__ void __launch_bounds__(kHistThreads) enc_hist_kernel(const __grid_constant__ EncArgs a) {
  __shared__ uint32_t s_hist[16];
  const int tid = threadIdx.x;
  if (tid < 16) s_hist[tid] = 0;
  __syncthreads();
  const int64_t row = blockIdx.y;
  const uint4 *src = reinterpret_cast<const uint4 *>(a.raw + row * a.n);
  const int64_t units = a.n / 16;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kHistThreads;
  unsigned long long lo = 0, hi = 0;
  int pending = 0;
  auto flush = [&]() {
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint32_t cl = static_cast<uint32_t>((lo >> (8 * b)) & 0xff);
      const uint32_t ch = static_cast<uint32_t>((hi >> (8 * b)) & 0xff);
      if (cl) atomicAdd(&s_hist[b], cl);
      if (ch) atomicAdd(&s_hist[8 + b], ch);
    }
    lo = hi = 0;
    pending = 0;
  };
  for (int64_t u = blockIdx.x * static_cast<int64_t>(kHistThreads) + tid; u < units; u += stride) {
    const uint4 v = src[u];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t e = (w[k] >> (8 * b + 3)) & 15;
        const unsigned long long inc = 1ull << (8 * (e & 7));
        lo += e < 8 ? inc : 0ull;
        hi += e < 8 ? 0ull : inc;
      }
    if (++pending == 15) flush();  // at most 240 counts per field
  }
  if (pending) flush();
  __syncthreads();
  if (tid < 16 && s_hist[tid]) atomicAdd(&row_scratch(a.scratch, row, a.G).hist[tid], s_hist[tid]);
}

// Plain Huffman lengths (codec.py:61-73): repeatedly merge the two smallest
// (count, tiebreak) entries; leaves have tiebreak = symbol, merged entries take
// 16, 17, ... in creation order.
__device__ void huffman_lengths(const double *counts, int *lengths) {
  double c[16];
  int tie[16];
  uint32_t members[16];
  int live = 16, next = 16;
  for (int i = 0; i < 16; ++i) {
    c[i] = counts[i];
    tie[i] = i;
    members[i] = 1u << i;
    lengths[i] = 0;
  }
  while (live > 1) {
    int a = 0;
    for (int i = 1; i < live; ++i)
      if (c[i] < c[a] || (c[i] == c[a] && tie[i] < tie[a])) a = i;
    const double ca = c[a];
    const uint32_t ma = members[a];
    c[a] = c[live - 1], tie[a] = tie[live - 1], members[a] = members[live - 1];
    --live;
    int b = 0;
    for (int i = 1; i < live; ++i)
      if (c[i] < c[b] || (c[i] == c[b] && tie[i] < tie[b])) b = i;
    const double cb = c[b];
    const uint32_t mb = members[b];
    c[b] = c[live - 1], tie[b] = tie[live - 1], members[b] = members[live - 1];
    --live;
    const uint32_t m = ma | mb;
    for (int s = 0; s < 16; ++s) lengths[s] += (m >> s) & 1;
    c[live] = ca + cb;
    tie[live] = next++;
    members[live] = m;
    ++live;
  }
}

// 2. Code lengths (codec.py:76-87: raise rare counts to sum / 2^(LIMIT-k) until
// every length fits LIMIT; the same float64 operations in the same order),
// canonical codes in (length, symbol) order stored bit-reversed
// (codec.py:90-106), and the LUT (codec.py:107-114).  One warp per row.
__global__ void __launch_bounds__(32) enc_code_kernel(const __grid_constant__ EncArgs a) {
  __shared__ uint32_t s_tab[16];
  const int lane = threadIdx.x;
  const int64_t row = blockIdx.x;
  RowScratch rs = row_scratch(a.scratch, row, a.G);
  if (lane == 0) {
    double counts[16];
    for (int i = 0; i < 16; ++i) {
      const uint32_t h = rs.hist[i];
      counts[i] = static_cast<double>(h > 1 ? h : 1);
    }
    int len[16];
    for (int k = 0;; ++k) {
      if (k > 0) {
        double sum = 0;
        for (int i = 0; i < 16; ++i) sum += counts[i];
        const double floor_ = sum / static_cast<double>(1 << (kLimit - k));
        for (int i = 0; i < 16; ++i) counts[i] = counts[i] > floor_ ? counts[i] : floor_;
      }
      huffman_lengths(counts, len);
      int mx = 0;
      for (int i = 0; i < 16; ++i) mx = len[i] > mx ? len[i] : mx;
      if (mx <= kLimit) break;
    }
    int order[16];
    for (int i = 0; i < 16; ++i) order[i] = i;
    for (int i = 1; i < 16; ++i)
      for (int j = i; j > 0 && (len[order[j]] < len[order[j - 1]] ||
                                (len[order[j]] == len[order[j - 1]] && order[j] < order[j - 1]));
           --j) {
        const int t = order[j];
        order[j] = order[j - 1];
        order[j - 1] = t;
      }
    uint32_t canon[16];
    uint32_t cc = 0;
    for (int i = 0; i < 16; ++i) {
      const int s = order[i];
      if (i) cc = (cc + 1) << (len[s] - len[order[i - 1]]);
      canon[s] = cc;
    }
    unsigned long long lens = 0;
    for (int s = 0; s < 16; ++s) {
      const uint32_t code = __brev(canon[s]) >> (32 - len[s]);
      s_tab[s] = code | (static_cast<uint32_t>(len[s]) << 16);
      rs.tab[s] = s_tab[s];
      lens |= static_cast<unsigned long long>(len[s]) << (4 * s);
    }
    *rs.lens = lens;
  }
  __syncwarp();
  // LUT entry x = (s << 4) | len for the symbol whose code is the low len bits of x.
  uint8_t *lut = a.luts + row * kLutBytes;
  for (int x = lane; x < kLutBytes; x += 32) {
    uint8_t v = 0;
    for (int s = 0; s < 16; ++s) {
      const uint32_t t = s_tab[s], len = t >> 16, code = t & 0xffff;
      if ((static_cast<uint32_t>(x) & ((1u << len) - 1)) == code) v = static_cast<uint8_t>((s << 4) | len);
    }
    lut[x] = v;
  }
}

// Code length of the exponent of byte x from the packed 4-bit lengths.
__device__ __forceinline__ uint32_t len_of(unsigned long long lens, uint32_t x) {
  return static_cast<uint32_t>(lens >> (4 * ((x >> 3) & 15))) & 15;
}

// 3. Words per group: lane l of group g holds values [(32g+l)*chunk, +chunk);
// its refill count is (bits before its last symbol + LIMIT-1) / 32 + 1
// (codec.py:150-156).
__global__ void __launch_bounds__(kWarpsPerBlock * 32) enc_count_kernel(const __grid_constant__ EncArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = blockIdx.y;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + warp;
  if (g >= a.G) return;
  RowScratch rs = row_scratch(a.scratch, row, a.G);
  const unsigned long long lens = *rs.lens;
  const uint2 *v = reinterpret_cast<const uint2 *>(a.raw + row * a.n + (g * 32 + lane) * a.chunk);
  uint32_t total = 0, last = 0;
  for (int64_t m = 0; m < a.chunk / 8; ++m) {
    const uint2 q = v[m];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      last = len_of(lens, (b < 4 ? q.x : q.y) >> (8 * (b & 3)));
      total += last;
    }
  }
  const uint32_t nw = (total - last + (kLimit - 1)) / 32 + 1;
  uint32_t sum = __reduce_add_sync(kFull, nw);
  if (lane == 0) rs.gw[g] = static_cast<int32_t>(sum);
}

// 4. gstart = exclusive scan of the group word counts; record size; the header
// (int32 gstart[G+1], codec.py:182-187) and a zeroed tail when the row fits.
__global__ void __launch_bounds__(kScanThreads) enc_scan_kernel(const __grid_constant__ EncArgs a) {
  using Scan = cub::BlockScan<long long, kScanThreads>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ long long s_carry;
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  RowScratch rs = row_scratch(a.scratch, row, a.G);
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int64_t g0 = 0; g0 < a.G; g0 += kScanThreads) {
    const int64_t g = g0 + tid;
    const long long x = g < a.G ? rs.gw[g] : 0;
    long long excl, agg;
    Scan(tmp).ExclusiveSum(x, excl, agg);
    const long long carry = s_carry;
    if (g < a.G) rs.gstart[g] = static_cast<int32_t>(carry + excl);
    __syncthreads();
    if (tid == 0) s_carry = carry + agg;
    __syncthreads();
  }
  const long long total = s_carry;
  const int64_t head = 4 * (a.G + 1) + a.n / 2;
  const int64_t nbytes = head + 4 * total;
  if (tid == 0) {
    rs.gstart[a.G] = static_cast<int32_t>(total);
    a.used[row] = nbytes;
  }
  if (nbytes > a.pitch) return;
  uint8_t *rec = a.records + row * a.pitch;
  int32_t *hdr = reinterpret_cast<int32_t *>(rec);
  for (int64_t g = tid; g < a.G; g += kScanThreads) hdr[g] = rs.gstart[g];
  if (tid == 0) hdr[a.G] = static_cast<int32_t>(total);
  for (int64_t i = nbytes + tid; i < a.pitch; i += kScanThreads) rec[i] = 0;
}

// Sign/mantissa nibble of byte x: (x >> 7) << 3 | (x & 7).
__device__ __forceinline__ uint32_t nib_of(uint32_t x) { return ((x >> 4) & 8) | (x & 7); }

// 5. Nibbles and Huffman words of one group per warp.
__global__ void __launch_bounds__(kWarpsPerBlock * 32) enc_emit_kernel(const __grid_constant__ EncArgs a) {
  __shared__ uint32_t s_code[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = blockIdx.y;
  RowScratch rs = row_scratch(a.scratch, row, a.G);
  if (threadIdx.x < 16) s_code[threadIdx.x] = rs.tab[threadIdx.x] & 0xffff;
  __syncthreads();
  const int64_t g = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + warp;
  if (g >= a.G) return;
  const int64_t head = 4 * (a.G + 1) + a.n / 2;
  if (head + 4 * static_cast<int64_t>(rs.gstart[a.G]) > a.pitch) return;  // does not fit
  const unsigned long long lens = *rs.lens;
  uint8_t *rec = a.records + row * a.pitch;
  uint32_t *nib = reinterpret_cast<uint32_t *>(rec + 4 * (a.G + 1));
  uint32_t *words = reinterpret_cast<uint32_t *>(rec + head);
  const int64_t M = a.chunk / 8;
  const uint2 *v = reinterpret_cast<const uint2 *>(a.raw + row * a.n + (g * 32 + lane) * a.chunk);
  const unsigned lt = lanemask_lt();
  uint32_t rp = static_cast<uint32_t>(rs.gstart[g]);  // next word slot of the group
  uint32_t slot0 = 0, slot1 = 0;                       // slots of words wk and wk + 1
  uint32_t refills = 0, wk = 0;
  int32_t before = 0;                                  // bits before the current symbol
  unsigned long long acc = 0;                          // bits of word wk onwards
  uint32_t accbits = 0;
  for (int64_t m = 0; m < M; ++m) {
    const uint2 q = v[m];  // values 8m .. 8m+7 of this lane
    uint32_t nw = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint32_t x = (b < 4 ? q.x : q.y) >> (8 * (b & 3));
      nw |= nib_of(x) << (4 * b);  // byte j = value 2j | value 2j+1 << 4
      // Refill before this symbol (the decoder's rule), slots in lane order.
      const bool need = static_cast<int32_t>(32 * refills) - before < kLimit;
      const unsigned bal = __ballot_sync(kFull, need);
      if (need) {
        const uint32_t slot = rp + __popc(bal & lt);
        if (refills & 1) slot1 = slot;
        else slot0 = slot;
        ++refills;
      }
      rp += __popc(bal);
      const uint32_t e = (x >> 3) & 15, len = static_cast<uint32_t>(lens >> (4 * e)) & 15;
      acc |= static_cast<unsigned long long>(s_code[e]) << accbits;
      accbits += len;
      before += static_cast<int32_t>(len);
      if (accbits >= 32) {  // word wk complete; its slot was handed out before its first bit
        words[(wk & 1) ? slot1 : slot0] = static_cast<uint32_t>(acc);
        acc >>= 32;
        accbits -= 32;
        ++wk;
      }
    }
    nib[(g * M + m) * 32 + lane] = nw;  // (group, word, lane) order, codec.py:140-143
  }
  // The last words: the partial one, then zeros up to the lane's refill count.
  while (wk < refills) {
    words[(wk & 1) ? slot1 : slot0] = static_cast<uint32_t>(acc);
    acc >>= 32;
    ++wk;
  }
}

}  // namespace
}  // namespace xp

using namespace xp;

extern "C" int64_t xp_encode_scratch_bytes(int64_t rows, int64_t n, int64_t chunk) {
  if (rows < 0 || n <= 0 || chunk < 8 || chunk % 8 || n % (32 * chunk)) return -1;
  return rows * row_scratch_bytes(n / (32 * chunk));
}

extern "C" int xp_encode_rows(const void *raw, int64_t rows, int64_t n, int64_t pitch,
                              int64_t chunk, void *records, void *luts, int64_t *used,
                              void *scratch, int64_t scratch_bytes, void *stream) {
  if (rows < 0 || chunk < 8 || chunk % 8 || n <= 0 || n % (32 * chunk) || pitch <= 0)
    return XP_EINVAL;
  if (rows == 0) return XP_OK;
  const int64_t G = n / (32 * chunk);
  if (!raw || !records || !luts || !used || !scratch || !aligned(raw, 16) ||
      !aligned(records, 4) || pitch % 4 || !aligned(scratch, 256) ||
      scratch_bytes < rows * row_scratch_bytes(G) || rows > 65535 || G > INT32_MAX / 4)
    return XP_EINVAL;
  EncArgs a{static_cast<const uint8_t *>(raw), rows, n, pitch, chunk, G,
            static_cast<uint8_t *>(records), static_cast<uint8_t *>(luts), used,
            static_cast<unsigned char *>(scratch)};
  cudaStream_t s = as_stream(stream);
  // One clear of the batch's scratch (the histograms accumulate by atomics).
  cudaError_t err = cudaMemsetAsync(scratch, 0, static_cast<size_t>(rows * row_scratch_bytes(G)), s);
  if (err != cudaSuccess) return static_cast<int>(err);
  enc_hist_kernel<<<dim3(kHistBlocksPerRow, static_cast<unsigned>(rows)), kHistThreads, 0, s>>>(a);
  enc_code_kernel<<<static_cast<unsigned>(rows), 32, 0, s>>>(a);
  const unsigned gb = static_cast<unsigned>((G + kWarpsPerBlock - 1) / kWarpsPerBlock);
  enc_count_kernel<<<dim3(gb, static_cast<unsigned>(rows)), kWarpsPerBlock * 32, 0, s>>>(a);
  enc_scan_kernel<<<static_cast<unsigned>(rows), kScanThreads, 0, s>>>(a);
  enc_emit_kernel<<<dim3(gb, static_cast<unsigned>(rows)), kWarpsPerBlock * 32, 0, s>>>(a);
  return launch_status();
}
