// Expansion of Huffman-compressed fp8 rows (staging -> VRAM slab).
//
// Record format and decode rule: monochromegane/vllm-expert-pager
// src/vllm_expert_pager/codec.py:1-41 (layout) and codec.py:204-289 (the Triton
// decoder).  A row of N values is split into groups of 32 lanes x chunk values;
// lane l of group g decodes values [(32g+l)*chunk, (32g+l+1)*chunk).  Each lane
// keeps a 64-bit bit buffer and, before every symbol, refills one 32-bit word
// when fewer than LIMIT=9 bits remain; lanes refilling at the same symbol
// index take consecutive words in lane order, starting at the group's first
// word gstart[g].  The 16 exponent symbols use canonical, bit-reversed codes
// of at most 9 bits looked up in a 512-entry LUT (sym << 4 | len); output byte
// = (s & 8) << 4 | sym << 3 | (s & 7) with s the stored sign/mantissa nibble.
//
// B200 mapping: one warp per group, four groups per CTA.
//  * The group's Huffman words are copied into shared memory first (cp.async,
//    16 bytes per lane per step, zero-filled past the record end).  Refilling
//    lanes then read consecutive words (ballot + popc give each its slot), so
//    a refill is one conflict-free shared load.  A group larger than the
//    per-warp buffer (flat exponent histograms only) takes a slower path that
//    streams the words through a register window.
//  * One unconditional lookup in the 512-byte LUT per symbol (the table is
//    512-byte aligned, so its address is one AND/OR of the window).  A two-level
//    lookup (a conflict-free 128-byte table for codes up to 7 bits, then a
//    predicated load of the full table) measured 12 % slower: the predicated
//    load stays on the symbol-to-symbol chain even when no lane takes it.
//  * Exponent bits of 4 symbols are summed into one word with one multiply-add
//    each (the bit fields do not overlap) and masked once; sign/mantissa
//    nibbles are spread to bytes with six bit operations per 4 values.
//  * Each lane stores 16 bytes per 16 symbols; nibble words are loaded two
//    iterations ahead and prefetched into L2 eight iterations ahead.
#include "common.cuh"

namespace xp {
namespace {

constexpr int kWarps = 4;
constexpr int kLimit = 9;
constexpr int kLutBytes = 512;
// Per-warp shared buffer for a group's Huffman words, in words: sized per launch
// from the records' pitch (see stage_words_for), within these bounds.
constexpr int64_t kStageMin = 1024, kStageMax = 4096;
constexpr unsigned kFull = 0xffffffffu;

struct DName {
  const uint8_t *stg;
  int64_t P;  // record (pitch) bytes
  uint8_t *dst;
  int64_t N;  // raw row bytes
  int64_t G;  // groups per row
};

struct DecodeArgs {
  const int64_t *todo;
  int64_t K;
  const int64_t *dst_row, *cache_row;
  const uint8_t *lut;  // [E][2][512]
  DName n[2];
  const int64_t *skip;
  int64_t chunk;
  int64_t stage_words;  // per-warp word buffer (multiple of 4)
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, int src_bytes) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Four sign/mantissa nibbles (x: bits 0..15) -> bytes (s & 7) | (s & 8) << 4.
__device__ __forceinline__ uint32_t spread(uint32_t x) {
  uint32_t t = (x | (x << 8)) & 0x00FF00FFu;
  t = (t | (t << 4)) & 0x0F0F0F0Fu;
  return (t & 0x07070707u) | ((t << 4) & 0x80808080u);
}

// One symbol step for lane state (buf, level): refill (warp-collective), look
// up, consume; returns the LUT entry.  Written in PTX, without branches.
// Shared-memory addresses are 32-bit: rp (the next unread word of the staged
// stream) and lut (512 B, 512-aligned).  The refilling lanes' word is the
// popc(bal & lt)-th after rp; rp is clamped to cap after each advance, off the
// symbol-to-symbol chain, so that rp + 4 * 31 stays inside the warp's buffer
// (a refilling lane of a valid record never leaves its group's words, which
// end at least 32 words before the buffer's end); buf |= w << level is one wide
// multiply-add because the new bits lie above level; the LUT address is the
// table's base OR the low 9 bits of the buffer.
__device__ __forceinline__ uint32_t step_staged(uint64_t &buf, int &level, uint32_t &rp,
                                                uint32_t cap, uint32_t lut,
                                                unsigned lt) {
  uint32_t ent;
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      ".reg .b32 bal, t, c, a, w, m, n, x, len;\n\t"
      "setp.lt.s32 p, %1, 9;\n\t"
      "vote.sync.ballot.b32 bal, p, 0xffffffff;\n\t"
      "and.b32 t, bal, %4;\n\t"
      "popc.b32 c, t;\n\t"
      "mad.lo.u32 a, c, 4, %2;\n\t"
      "ld.shared.u32 w, [a];\n\t"
      "shl.b32 m, 1, %1;\n\t"
      "selp.b32 m, m, 0, p;\n\t"
      "mad.wide.u32 %0, w, m, %0;\n\t"
      "@p add.s32 %1, %1, 32;\n\t"
      "popc.b32 n, bal;\n\t"
      "mad.lo.u32 %2, n, 4, %2;\n\t"
      "min.u32 %2, %2, %5;\n\t"
      "cvt.u32.u64 x, %0;\n\t"
      "and.b32 t, x, 511;\n\t"
      "or.b32 t, t, %6;\n\t"
      "ld.shared.u8 %3, [t];\n\t"
      "and.b32 len, %3, 15;\n\t"
      "shr.b64 %0, %0, len;\n\t"
      "sub.s32 %1, %1, len;\n\t"
      "}"
      : "+l"(buf), "+r"(level), "+r"(rp), "=r"(ent)
      : "r"(lt), "r"(cap), "r"(lut));
  return ent;
}

// Slow path for a group whose words do not fit the shared buffer: a 96-word
// register window slid with coalesced loads, words handed out by shuffles.
__device__ void decode_group_window(const uint32_t *huff, int64_t wbase, int64_t rend,
                                    const uint32_t *nib, uint8_t *out_row, int64_t chunk,
                                    const uint8_t *L, int lane) {
  auto ld = [&](int64_t idx) -> uint32_t {
    return (idx >= 0 && idx < rend) ? __ldg(huff + idx) : 0u;
  };
  uint32_t w0 = ld(wbase + lane), w1 = ld(wbase + 32 + lane), w2 = ld(wbase + 64 + lane);
  uint64_t *out = reinterpret_cast<uint64_t *>(out_row);
  uint64_t buf = 0;
  int level = 0, rel = 0;
  const unsigned lt = lanemask_lt();
  for (int64_t m = 0; m < chunk / 8; ++m) {
    const uint32_t nw = __ldg(nib + m * 32 + lane);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const bool need = level < kLimit;
      const unsigned bal = __ballot_sync(kFull, need);
      if (bal) {
        const int pos = rel + __popc(bal & lt);
        const uint32_t a0 = __shfl_sync(kFull, w0, pos & 31);
        const uint32_t a1 = __shfl_sync(kFull, w1, pos & 31);
        if (need) {
          buf |= static_cast<uint64_t>(pos < 32 ? a0 : a1) << level;
          level += 32;
        }
        rel += __popc(bal);
        if (rel >= 32) {
          rel -= 32;
          wbase += 32;
          w0 = w1;
          w1 = w2;
          w2 = ld(wbase + 64 + lane);
        }
      }
      const uint32_t ent = L[buf & (kLutBytes - 1)];
      const uint32_t len = ent & 15;
      buf >>= len;
      level -= static_cast<int>(len);
      const uint32_t s = (nw >> (4 * k)) & 15;
      const uint32_t byte = ((s & 8) << 4) | ((ent >> 4) << 3) | (s & 7);
      if (k < 4) lo |= byte << (8 * k);
      else hi |= byte << (8 * (k - 4));
    }
    out[m] = (static_cast<uint64_t>(hi) << 32) | lo;
  }
}

__global__ void __launch_bounds__(kWarps * 32) decode_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(16) uint32_t s_words[];  // [kWarps][stage_words]
  __shared__ __align__(512) uint8_t s_lut[kWarps][kLutBytes];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t j = blockIdx.y;
  const int64_t gg = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (gg >= a.n[0].G + a.n[1].G) return;
  const int which = gg < a.n[0].G ? 0 : 1;
  const DName &n = a.n[which];
  const int64_t g = which ? gg - a.n[0].G : gg;
  const int64_t chunk = a.chunk, G = n.G;
  const uint8_t *rec = n.stg + j * n.P;
  const int64_t head = 4 * (G + 1);
  const int32_t *hdr = reinterpret_cast<const int32_t *>(rec);
  const int64_t huff_w = (head + n.N / 2) / 4;  // first Huffman word, from the record start
  const int64_t rec_w = n.P / 4;
  // The prologue takes three round trips to global memory.  First: the todo
  // entry and the group's word range [gstart[g], gstart[g+1]) from the header of
  // staging row j (row j exists for every todo index).
  const int64_t e = a.todo[j];
  int64_t w_begin = hdr[g], w_end = hdr[g + 1];
  if (e < 0) return;
  // Second, in flight together: the skip list (one entry per lane), the
  // expert's cache and destination rows and its LUT.
  const int64_t sk0 = (a.skip && lane < a.K) ? a.skip[lane] : -1;
  const int64_t crow = a.cache_row[e];
  int64_t dst_row = a.dst_row[e];
  const uint4 lut_v = reinterpret_cast<const uint4 *>(a.lut + (e * 2 + which) * kLutBytes)[lane];
  bool skipped = __any_sync(kFull, sk0 == e);
  if (a.skip)
    for (int64_t k0 = 32; k0 < a.K; k0 += 32) {
      const int64_t k = k0 + lane;
      skipped |= __any_sync(kFull, k < a.K && a.skip[k] == e);
    }
  // Skipped, or copied raw from the cache slab: the staging row holds no record
  // of this expert, and nothing past its header is read.
  if (skipped || crow >= 0) return;
  // Third: the group's words, clamped to the record (a corrupt header cannot
  // move a read outside row j).
  const int64_t wmax = rec_w - huff_w;
  w_end = w_end < 0 ? 0 : (w_end > wmax ? wmax : w_end);
  w_begin = w_begin < 0 ? 0 : (w_begin > w_end ? w_end : w_begin);
  uint8_t *L = s_lut[warp];
  reinterpret_cast<uint4 *>(L)[lane] = lut_v;
  dst_row = dst_row > 0 ? dst_row : 0;
  const uint32_t *nib = reinterpret_cast<const uint32_t *>(rec + head) + g * (chunk / 8) * 32;
  uint8_t *out_row = n.dst + dst_row * n.N + (g * 32 + lane) * chunk;
  // The words go to shared memory in 16-byte units aligned to the record
  // (4096-aligned rows, so record word 4u is 16-byte aligned).
  const int64_t a_begin = huff_w + w_begin, a_end = huff_w + w_end;
  const int64_t a0 = a_begin & ~int64_t(3);
  const int64_t units = (a_end - a0 + 3) / 4;
  const bool staged = units * 4 + 32 <= a.stage_words && (chunk / 8) % 2 == 0;
  if (!staged) {
    __syncwarp();
    decode_group_window(reinterpret_cast<const uint32_t *>(rec) + huff_w, w_begin,
                        w_end, nib, out_row, chunk, L, lane);
    return;
  }
  uint32_t *words = s_words + warp * a.stage_words;
  for (int64_t u = lane; u < units; u += 32) {
    const int64_t w = a0 + 4 * u;
    int64_t bytes = (rec_w - w) * 4;
    bytes = bytes < 0 ? 0 : (bytes > 16 ? 16 : bytes);
    cp_async16(words + 4 * u, rec + 4 * (bytes > 0 ? w : 0), static_cast<int>(bytes));
  }
  cp_async_wait_all();
  __syncwarp();

  const unsigned lt = lanemask_lt();
  uint64_t buf = 0;
  int level = 0;
  const uint32_t sw = static_cast<uint32_t>(__cvta_generic_to_shared(words));
  uint32_t rp = sw + static_cast<uint32_t>(4 * (a_begin - a0));
  const uint32_t cap = sw + static_cast<uint32_t>(4 * (a.stage_words - 32));
  const uint32_t sl = static_cast<uint32_t>(__cvta_generic_to_shared(L));
  const int64_t steps = chunk / 8;
  // Nibble words are loaded into registers two iterations ahead, and their
  // 128-byte lines are prefetched into L2 sixteen words (eight iterations) ahead,
  // which hides the HBM latency that the register prefetch alone leaves exposed
  // (7 % of the kernel at 8 rows per launch).  The index is clamped (steps is even
  // and at least 2) rather than the load predicated, so that no select consumes
  // a load right after it is issued.
  const int64_t last = steps - 1;
  for (int64_t i = lane; i < 16 && i <= last; i += 32)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(nib + i * 32));
  uint32_t q0 = __ldg(nib + lane);
  uint32_t q1 = __ldg(nib + 32 + lane);
  uint32_t q2 = __ldg(nib + (2 < last ? 2 : last) * 32 + lane);
  uint32_t q3 = __ldg(nib + (3 < last ? 3 : last) * 32 + lane);
  uint4 *out = reinterpret_cast<uint4 *>(out_row);
  // Unrolled twice so that consecutive 16-byte stores take different registers:
  // the next iteration's results need not wait for the store to read its own.
#pragma unroll 2
  for (int64_t m = 0; m < steps; m += 2) {
    uint32_t lohi[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t nw = h ? q1 : q0;
      uint32_t acc_lo, acc_hi;
      {
        uint32_t ent = step_staged(buf, level, rp, cap, sl, lt);
        acc_lo = ent >> 1;
#pragma unroll
        for (int k = 1; k < 4; ++k) {
          ent = step_staged(buf, level, rp, cap, sl, lt);
          acc_lo += ent << (8 * k - 1);
        }
        ent = step_staged(buf, level, rp, cap, sl, lt);
        acc_hi = ent >> 1;
#pragma unroll
        for (int k = 1; k < 4; ++k) {
          ent = step_staged(buf, level, rp, cap, sl, lt);
          acc_hi += ent << (8 * k - 1);
        }
      }
      lohi[2 * h] = (acc_lo & 0x78787878u) | spread(nw & 0xFFFFu);
      lohi[2 * h + 1] = (acc_hi & 0x78787878u) | spread(nw >> 16);
    }
    out[m / 2] = make_uint4(lohi[0], lohi[1], lohi[2], lohi[3]);
    q0 = q2;
    q1 = q3;
    if (lane < 2 && m + 16 + lane <= last)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(nib + (m + 16 + lane) * 32));
    q2 = __ldg(nib + (m + 4 < last ? m + 4 : last) * 32 + lane);
    q3 = __ldg(nib + (m + 5 < last ? m + 5 : last) * 32 + lane);
  }
}

// Words per warp buffer for records of pitch P holding N values: the mean
// Huffman words per group when the record is full, plus an eighth for groups
// above the mean and the 32 words of refill slack; groups larger than that take
// the register-window path.  A smaller buffer fits more CTAs per SM.
int64_t stage_words_for(int64_t P, int64_t N, int64_t chunk) {
  const int64_t G = N / (32 * chunk);
  const int64_t huff = (P - 4 * (G + 1) - N / 2) / 4;
  const int64_t mean = (huff + G - 1) / G;
  int64_t w = mean + mean / 8 + 32;
  w = (w + 3) / 4 * 4;
  return w < kStageMin ? kStageMin : (w > kStageMax ? kStageMax : w);
}

}  // namespace
}  // namespace xp

using namespace xp;

extern "C" int xp_decode_rows(const int64_t *todo, int64_t K, const int64_t *dst_row,
                              const int64_t *cache_row, const uint8_t *lut, const void *stg0,
                              int64_t P0, void *dst0, int64_t N0, const void *stg1, int64_t P1,
                              void *dst1, int64_t N1, const int64_t *skip, int64_t chunk,
                              void *stream) {
  if (K < 0 || K > 65535 || chunk < 8 || chunk % 8) return XP_EINVAL;
  if (K == 0) return XP_OK;
  if (!todo || !dst_row || !cache_row || !lut || !aligned(lut, 16)) return XP_EINVAL;
  DecodeArgs a{};
  a.todo = todo;
  a.K = K;
  a.dst_row = dst_row;
  a.cache_row = cache_row;
  a.lut = lut;
  a.skip = skip;
  a.chunk = chunk;
  const void *stgs[2] = {stg0, stg1};
  void *dsts[2] = {dst0, dst1};
  const int64_t Ps[2] = {P0, P1}, Ns[2] = {N0, N1};
  for (int i = 0; i < 2; ++i) {
    const int64_t N = Ns[i], P = Ps[i];
    if (N <= 0 || N % (32 * chunk) || P % 16 || P < 4 * (N / (32 * chunk) + 1) + N / 2)
      return XP_EINVAL;
    // Records start on 16-byte boundaries (cp.async); the 16-byte output stores
    // need 16-byte aligned lane chunks.
    if (!stgs[i] || !dsts[i] || !aligned(stgs[i], 16) || !aligned(dsts[i], 16))
      return XP_EINVAL;
    a.n[i] = DName{static_cast<const uint8_t *>(stgs[i]), P, static_cast<uint8_t *>(dsts[i]), N,
                   N / (32 * chunk)};
  }
  const int64_t sw0 = stage_words_for(P0, N0, chunk), sw1 = stage_words_for(P1, N1, chunk);
  a.stage_words = sw0 > sw1 ? sw0 : sw1;
  const size_t smem = static_cast<size_t>(kWarps * 4 * a.stage_words);
  if (smem > 48 * 1024) {
    cudaError_t err = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return static_cast<int>(err);
  }
  const int64_t groups = a.n[0].G + a.n[1].G;
  dim3 grid(static_cast<unsigned>((groups + kWarps - 1) / kWarps), static_cast<unsigned>(K));
  decode_kernel<<<grid, kWarps * 32, smem, as_stream(stream)>>>(a);
  return launch_status();
}
