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
//  * The group's Huffman words stream through a 4 KiB shared-memory ring per
//    warp, filled by cp.async half a ring ahead of the reader; refilling lanes
//    read consecutive words (ballot + popc give each its slot), one
//    conflict-free shared load.  The ring (instead of staging a whole group,
//    ~7.3 KiB) lets 10 CTAs share an SM.
//  * One unconditional lookup in the 512-byte LUT per symbol (the table is
//    512-byte aligned, so its address is one AND/OR of the window).
//  * The kernel is bound by the integer ALU pipe (half rate: one warp
//    instruction per two cycles per scheduler) and, in small launches, by the
//    symbol-to-symbol dependency chain.  Exponent bits of 4 symbols are summed
//    with multiply-adds and sign/mantissa nibbles spread with multiplies, both on
//    the FMA pipe; one select merges them.
//  * Small launches (at most 12 warps per SM) decide each symbol's refill one
//    symbol early from a length-only lookup of the pre-insert buffer, which
//    takes the ballot -> word-load latency off the per-symbol chain at the cost
//    of a second lookup; larger launches are throughput-bound and use the plain
//    step.
//  * Each lane stores 16 bytes per 16 symbols; nibble words are loaded two
//    iterations ahead and prefetched into L2 eight iterations ahead.
#include <atomic>

#include "common.cuh"

namespace xp {
namespace {

constexpr int kWarps = 4;
constexpr int kLimit = 9;
constexpr int kLutBytes = 512;
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
};

// Path for chunk sizes whose 8-value blocks per lane are odd in number (the
// main loop stores 16 values per lane at a time): a 96-word register window
// slid with coalesced loads, words handed out by shuffles.
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

// Integer helpers that keep work off the integer ALU pipe, which bounds this
// kernel (one ALU warp instruction per two cycles per scheduler): multiplies
// run on the FMA pipe.
__device__ __forceinline__ uint32_t mad_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t mul_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.lo.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Bitwise select: (a & m) | (b & ~m), one three-input logic op.
__device__ __forceinline__ uint32_t bitsel(uint32_t a, uint32_t b, uint32_t m) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(d) : "r"(a), "r"(b), "r"(m));
  return d;
}

// Output bytes of 4 symbols: acc = e0 + e1 << 8 + e2 << 16 + e3 << 24 (LUT
// entries sym << 4 | len), x = their 4 sign/mantissa nibbles (bits 0..15).
// Byte k = (s & 8) << 4 | sym << 3 | (s & 7).  The nibbles are spread to one
// per byte with two multiplies whose partial products do not collide inside
// the kept bits (x & 0x0F0F times 257 puts n0, n2 at bytes 0, 2; x & 0xF0F0
// times 4112 puts n1, n3 at bytes 1, 3), t * 17 copies each nibble to the high
// half of its byte, and one select merges the exponent field (acc >> 1 has
// sym at bits 3..6 of each byte) with the sign and mantissa bits.
__device__ __forceinline__ uint32_t merge4(uint32_t acc, uint32_t x) {
  const uint32_t t = bitsel(mul_u32(x & 0x0F0Fu, 257u), mul_u32(x & 0xF0F0u, 4112u), 0x001F001Fu);
  return bitsel(acc >> 1, mul_u32(t, 17u), 0x78787878u);
}

// Word ring.  Each warp streams its group's Huffman words through a 4 KiB
// shared-memory ring (1,024 words), filled half by half (2 KiB = 128 cp.async
// units of 16 bytes, 4 per lane) as the read offset enters the newest half;
// a half in flight is waited for only when the reader comes within 1 KiB of
// it.  A valid record's refills advance the reader by at most 6 words per lane
// per 16 symbols (a lane refills at most once every 3 symbols), 768 bytes, so
// a fill issued half a ring ahead has about 70 symbol steps to land.  Word
// addresses are (offset & 4095) | base with a 4 KiB-aligned base, so no read
// leaves the ring whatever the record holds: a corrupt record can only decode
// to wrong bytes.
constexpr uint32_t kRing = 4096, kHalf = 2048;
// Dynamic shared memory per CTA: kWarps rings plus the slack that aligns them.
constexpr size_t kRingSmem = kWarps * kRing + kRing;

// One symbol step with ring-addressed refills.  nv = 8 - level: this symbol
// refills iff nv >= 0, and 0x100 >> nv is then 1 << level (0 otherwise: the
// shift count of a negative nv is clamped to 32), the multiplier that places
// the new word above the buffer's valid bits.  off is the byte offset of the
// next unread word in the group's stream (the ring slot is off mod 4 KiB).
__device__ __forceinline__ uint32_t step_ring(uint64_t &buf, int &nv, uint32_t &off,
                                              uint32_t base, uint32_t lut, unsigned lt) {
  uint32_t ent;
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      ".reg .b32 bal, t, c, a, w, m, n, x, len;\n\t"
      "setp.ge.s32 p, %1, 0;\n\t"
      "vote.sync.ballot.b32 bal, p, 0xffffffff;\n\t"
      "and.b32 t, bal, %4;\n\t"
      "popc.b32 c, t;\n\t"
      "mad.lo.u32 a, c, 4, %2;\n\t"
      "and.b32 a, a, 4095;\n\t"
      "or.b32 a, a, %5;\n\t"
      "ld.shared.u32 w, [a];\n\t"
      "shr.b32 m, 256, %1;\n\t"
      "mad.wide.u32 %0, w, m, %0;\n\t"
      "@p add.s32 %1, %1, -32;\n\t"
      "popc.b32 n, bal;\n\t"
      "mad.lo.u32 %2, n, 4, %2;\n\t"
      "cvt.u32.u64 x, %0;\n\t"
      "and.b32 t, x, 511;\n\t"
      "or.b32 t, t, %6;\n\t"
      "ld.shared.u8 %3, [t];\n\t"
      "and.b32 len, %3, 15;\n\t"
      "shr.b64 %0, %0, len;\n\t"
      "add.s32 %1, %1, len;\n\t"
      "}"
      : "+l"(buf), "+r"(nv), "+r"(off), "=r"(ent)
      : "r"(lt), "r"(base), "r"(lut));
  return ent;
}


// step_ring with the refill decision of the next symbol taken before this
// symbol's insert (the one-ahead pipeline of step_piped, ring-addressed): a
// lane that does not refill here knows this symbol's length from its current
// buffer, so the next symbol's ballot and word load need not wait for this
// symbol's insert and lookup.  Both lookups are issued first.  w is the word
// this lane takes at this symbol if it refills here (loaded one step before).
__device__ __forceinline__ uint32_t step_ring_piped(uint64_t &buf, int &nv, uint32_t &off,
                                                    uint32_t &w, uint32_t base, uint32_t lut,
                                                    uint32_t lenlut, unsigned lt) {
  uint32_t ent, wn;
  asm volatile(
      "{\n\t"
      ".reg .pred r, pn;\n\t"
      ".reg .b32 x, ia, la, t, bal, c, a, n, m, ib, len;\n\t"
      ".reg .b64 bi;\n\t"
      "setp.ge.s32 r, %1, 0;\n\t"
      "cvt.u32.u64 x, %0;\n\t"
      "and.b32 ia, x, 511;\n\t"
      "or.b32 ia, ia, %8;\n\t"
      "ld.shared.u8 la, [ia];\n\t"
      "shr.b32 m, 256, %1;\n\t"
      "mad.wide.u32 bi, %9, m, %0;\n\t"
      "cvt.u32.u64 x, bi;\n\t"
      "and.b32 ib, x, 511;\n\t"
      "or.b32 ib, ib, %7;\n\t"
      "ld.shared.u8 %3, [ib];\n\t"
      "add.s32 t, %1, la;\n\t"
      "setp.ge.and.s32 pn, t, 0, !r;\n\t"
      "vote.sync.ballot.b32 bal, pn, 0xffffffff;\n\t"
      "and.b32 c, bal, %5;\n\t"
      "popc.b32 c, c;\n\t"
      "mad.lo.u32 a, c, 4, %2;\n\t"
      "and.b32 a, a, 4095;\n\t"
      "or.b32 a, a, %6;\n\t"
      "ld.shared.u32 %4, [a];\n\t"
      "popc.b32 n, bal;\n\t"
      "mad.lo.u32 %2, n, 4, %2;\n\t"
      "@r add.s32 %1, %1, -32;\n\t"
      "and.b32 len, %3, 15;\n\t"
      "shr.b64 %0, bi, len;\n\t"
      "add.s32 %1, %1, len;\n\t"
      "}"
      : "+l"(buf), "+r"(nv), "+r"(off), "=&r"(ent), "=&r"(wn)
      : "r"(lt), "r"(base), "r"(lut), "r"(lenlut), "r"(w));
  w = wn;
  return ent;
}

__device__ __forceinline__ void cp_async16_s(uint32_t saddr, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gmem) : "memory");
}

// Copies stream bytes [lo, hi) (16-byte units; the caller keeps hi - lo at
// most one ring) of the group's words into their ring slots.
__device__ __forceinline__ void ring_fill(uint32_t base, const uint8_t *src, uint32_t lo,
                                          uint32_t hi, int lane) {
  for (uint32_t p = lo + 16u * lane; p < hi; p += 512u) cp_async16_s(base + (p & (kRing - 1)), src + p);
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <bool kPiped>
__global__ void __launch_bounds__(kWarps * 32) decode_ring_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t s_dyn[];  // kWarps rings of 4 KiB, 4 KiB-aligned
  __shared__ __align__(512) uint8_t s_lut[kWarps][kLutBytes];
  __shared__ __align__(512) uint8_t s_len[kPiped ? kWarps : 1][kLutBytes];  // lengths only
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
  const int64_t huff_w = (head + n.N / 2) / 4;
  const int64_t rec_w = n.P / 4;
  // Three global round trips: the todo entry and the
  // group's word range; the skip list, cache/destination rows and LUT; then
  // the group's first ring of words.
  const int64_t e = a.todo[j];
  int64_t w_begin = hdr[g], w_end = hdr[g + 1];
  if (e < 0) return;
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
  if (skipped || crow >= 0) return;
  const int64_t wmax = rec_w - huff_w;
  w_end = w_end < 0 ? 0 : (w_end > wmax ? wmax : w_end);
  w_begin = w_begin < 0 ? 0 : (w_begin > w_end ? w_end : w_begin);
  uint8_t *L = s_lut[warp];
  reinterpret_cast<uint4 *>(L)[lane] = lut_v;
  if (kPiped)
    reinterpret_cast<uint4 *>(s_len[warp])[lane] =
        make_uint4(lut_v.x & 0x0F0F0F0Fu, lut_v.y & 0x0F0F0F0Fu, lut_v.z & 0x0F0F0F0Fu,
                   lut_v.w & 0x0F0F0F0Fu);
  dst_row = dst_row > 0 ? dst_row : 0;
  const uint32_t *nib = reinterpret_cast<const uint32_t *>(rec + head) + g * (chunk / 8) * 32;
  uint8_t *out_row = n.dst + dst_row * n.N + (g * 32 + lane) * chunk;
  const int64_t a_begin = huff_w + w_begin, a_end = huff_w + w_end;
  const int64_t a0 = a_begin & ~int64_t(3);  // 16-byte aligned (records are 16-byte aligned)
  if ((chunk / 8) % 2) {
    __syncwarp();
    decode_group_window(reinterpret_cast<const uint32_t *>(rec) + huff_w, w_begin, w_end, nib,
                        out_row, chunk, L, lane);
    return;
  }
  // The stream: bytes [0, total) from record word a0, in 16-byte units (the
  // last unit ends inside the record: P and a0 are multiples of 16 bytes).
  const uint8_t *src = rec + 4 * a0;
  const uint32_t total = static_cast<uint32_t>((a_end - a0 + 3) / 4 * 16);
  const uint32_t dyn = static_cast<uint32_t>(__cvta_generic_to_shared(s_dyn));
  const uint32_t base = ((dyn + kRing - 1) & ~(kRing - 1)) + warp * kRing;
  uint32_t filled = total < kRing ? total : kRing;
  ring_fill(base, src, 0, filled, lane);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncwarp();
  bool pending = false;

  const unsigned lt = lanemask_lt();
  uint64_t buf = 0;
  int nv = 8;
  uint32_t off = static_cast<uint32_t>(4 * (a_begin - a0));
  const uint32_t sl = static_cast<uint32_t>(__cvta_generic_to_shared(L));
  const uint32_t sn = static_cast<uint32_t>(__cvta_generic_to_shared(s_len[kPiped ? warp : 0]));
  // Pipelined step: every lane refills at symbol 0 (level 0) and takes the
  // group's first 32 words in lane order.
  uint32_t w = 0;
  if (kPiped) {
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w) : "r"(base + ((off + 4u * lane) & (kRing - 1))));
    off += 128;
  }
  auto step = [&]() {
    return kPiped ? step_ring_piped(buf, nv, off, w, base, sl, sn, lt)
                  : step_ring(buf, nv, off, base, sl, lt);
  };
  const int64_t steps = chunk / 8;
  const int64_t last = steps - 1;
  for (int64_t i = lane; i < 16 && i <= last; i += 32)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(nib + i * 32));
  uint32_t q0 = __ldg(nib + lane);
  uint32_t q1 = __ldg(nib + 32 + lane);
  uint32_t q2 = __ldg(nib + (2 < last ? 2 : last) * 32 + lane);
  uint32_t q3 = __ldg(nib + (3 < last ? 3 : last) * 32 + lane);
  uint4 *out = reinterpret_cast<uint4 *>(out_row);
#pragma unroll 2
  for (int64_t m = 0; m < steps; m += 2) {
    // Ring upkeep, warp-uniform (off and filled are the same in every lane).
    if (filled < total && off + kHalf >= filled) {
      const uint32_t hi = filled + kHalf < total ? filled + kHalf : total;
      ring_fill(base, src, filled, hi, lane);
      filled = hi;
      pending = true;
    }
    if (pending && off + 1024 + kHalf >= filled) {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncwarp();
      pending = false;
    }
    uint32_t lohi[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t nw = h ? q1 : q0;
      uint32_t acc_lo = step();
#pragma unroll
      for (int k = 1; k < 4; ++k) acc_lo = mad_u32(step(), 1u << (8 * k), acc_lo);
      uint32_t acc_hi = step();
#pragma unroll
      for (int k = 1; k < 4; ++k) acc_hi = mad_u32(step(), 1u << (8 * k), acc_hi);
      lohi[2 * h] = merge4(acc_lo, nw & 0xFFFFu);
      lohi[2 * h + 1] = merge4(acc_hi, nw >> 16);
    }
    out[m / 2] = make_uint4(lohi[0], lohi[1], lohi[2], lohi[3]);
    q0 = q2;
    q1 = q3;
    if (lane < 2 && m + 16 + lane <= last)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(nib + (m + 16 + lane) * 32));
    q2 = __ldg(nib + (m + 4 < last ? m + 4 : last) * 32 + lane);
    q3 = __ldg(nib + (m + 5 < last ? m + 5 : last) * 32 + lane);
  }
  // Leave no copy in flight into shared memory at exit.
  asm volatile("cp.async.wait_group 0;" ::: "memory");
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
  const int64_t groups = a.n[0].G + a.n[1].G;
  // Launches of at most 12 warps per SM are latency-bound (three warps or
  // fewer per scheduler): they take the pipelined step.
  static std::atomic<int> sm_count[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return XP_EINVAL;
  int sms = sm_count[dev].load(std::memory_order_relaxed);
  if (sms == 0) {
    cudaError_t err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return static_cast<int>(err);
    sms = sms > 0 ? sms : 1;
    sm_count[dev].store(sms, std::memory_order_relaxed);
  }
  const bool piped = K * groups <= int64_t(12) * sms;
  dim3 grid(static_cast<unsigned>((groups + kWarps - 1) / kWarps), static_cast<unsigned>(K));
  auto kern = piped ? decode_ring_kernel<true> : decode_ring_kernel<false>;
  kern<<<grid, kWarps * 32, kRingSmem, as_stream(stream)>>>(a);
  return launch_status();
}
