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
//  * The group's Huffman words stream through a 2 KiB shared-memory ring per
//    warp, filled by cp.async half a ring ahead of the reader; refilling lanes
//    read consecutive words (ballot + popc give each its slot), one
//    conflict-free shared load.  The ring (instead of staging a whole group,
//    ~7.3 KiB) and a 48-register bound let 10 CTAs (40 warps) share an SM.
//  * Several symbols per ballot round (step_triple, step_pair; 8 symbols in
//    rounds of 3 + 3 + 2): a lane refills at most once in three consecutive
//    symbols, its refill symbol follows from length-only lookups of its current
//    buffer, and its word can be inserted above its valid bits before the
//    round's first symbol; so one round of ballots and one word load serves
//    two or three symbols, which cuts the refill work on the symbol-to-symbol
//    chain.
//  * One lookup in the 512-byte LUT per symbol (the table is 512-byte aligned,
//    so its address is one AND/OR of the window).
//  * Every instruction is integer work; the integer ALU pipe (one warp
//    instruction per two cycles per scheduler) is the busiest unit in large
//    launches.  Exponent bits of 4 symbols are summed with multiply-adds and
//    sign/mantissa nibbles spread with multiplies, both on the FMA pipe; one
//    select merges them.
//  * Each lane stores 16 bytes per 16 symbols; nibble words are loaded two
//    iterations ahead and prefetched into L2 eight iterations ahead.
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

// Word ring.  Each warp streams its group's Huffman words through a 2 KiB
// shared-memory ring (512 words), filled half by half (1 KiB = 64 cp.async
// units of 16 bytes, 2 per lane) as the read offset enters the newest half.
// A valid record's refills advance the reader by at most 6 words per lane per
// 16 symbols (a lane refills at most once every 3 symbols), kMaxAdvance = 768
// bytes, the only words whose values matter (lanes that do not refill read
// words they discard); so a half in flight is waited for, at the top of a
// 16-symbol iteration, only when the reader is within 768 bytes of it, which
// leaves a fill 256 bytes (~18 symbol steps) to land.  Word addresses are
// (offset & 2047) | base with a 2 KiB-aligned base, so no read leaves the ring
// whatever the record holds: a corrupt record can only decode to wrong bytes.
constexpr uint32_t kRing = 2048, kHalf = 1024;
#define XP_RING_MASK "2047"  // kRing - 1, spelled for the step functions' PTX
static_assert(kRing == 2048, "XP_RING_MASK spells kRing - 1");
// Most stream bytes a valid record's refills consume in 16 symbols: a lane
// refills at most once every 3 symbols, so 6 words per lane.
constexpr uint32_t kMaxAdvance = 6 * 32 * 4;
// Dynamic shared memory per CTA: kWarps rings plus the slack that aligns them.
constexpr size_t kRingSmem = kWarps * kRing + kRing;

// Two symbols per ballot round.  A lane that refills at symbol i cannot refill
// at i+1 (the refill leaves at least 23 bits after symbol i), so each lane
// refills at most once per pair, at i (level < 9) or at i+1 (level >= 9 and
// level - len_i < 9, len_i from a length-only lookup of the current buffer,
// which holds level >= 9 valid bits).  The pair's refills go in the format's
// order (all of symbol i's in lane order, then symbol i+1's): with C0 the
// ballot of lanes refilling at i and C1 that of lanes refilling at i or i+1
// (level + len_i < 9 + len_i, i.e. nv + len_i >= 0, which holds for every lane
// refilling at i as well), a lane refilling at slot k takes the word after
// popc(C_{k-1} | (C_k & lanes below it)) others (C_{-1} = 0), and the pair uses
// popc(C1) words; one shared load gives each refilling lane its word, and the
// word is inserted
// right above the lane's valid bits before symbol i: for a lane refilling at
// i+1 that is where the format puts it after symbol i's bits are consumed, and
// symbol i reads only bits below it.  The insert position is at most 23 bits,
// so the 64-bit buffer holds it; its multiplier 0x800000 >> (nv + 15) is
// 1 << level for level <= 23.  Returns the two LUT entries.
__device__ __forceinline__ void step_pair(uint64_t &buf, int &nv, uint32_t &off, uint32_t base,
                                          uint32_t lut, uint32_t lenlut, unsigned lt,
                                          uint32_t &e0, uint32_t &e1) {
  asm volatile(
      "{\n\t"
      ".reg .pred p0, ev;\n\t"
      ".reg .b32 x, ia, l0, t, b0, b1, n0, n1, mb, c, a, w, m, len;\n\t"
      "setp.ge.s32 p0, %1, 0;\n\t"
      "cvt.u32.u64 x, %0;\n\t"
      "and.b32 ia, x, 511;\n\t"
      "or.b32 ia, ia, %8;\n\t"
      "ld.shared.u8 l0, [ia];\n\t"
      "add.s32 t, %1, l0;\n\t"
      "setp.ge.s32 ev, t, 0;\n\t"
      "vote.sync.ballot.b32 b0, p0, 0xffffffff;\n\t"
      "vote.sync.ballot.b32 b1, ev, 0xffffffff;\n\t"
      "selp.b32 n0, 0, b0, p0;\n\t"
      "selp.b32 mb, b0, b1, p0;\n\t"
      "lop3.b32 mb, mb, n0, %5, 0xE4;\n\t"
      "popc.b32 c, mb;\n\t"
      "mad.lo.u32 a, c, 4, %2;\n\t"
      "and.b32 a, a, " XP_RING_MASK ";\n\t"
      "or.b32 a, a, %6;\n\t"
      "ld.shared.u32 w, [a];\n\t"
      "popc.b32 n1, b1;\n\t"
      "mad.lo.u32 %2, n1, 4, %2;\n\t"
      "add.s32 t, %1, 15;\n\t"
      "shr.b32 m, 8388608, t;\n\t"
      "@ev mad.wide.u32 %0, w, m, %0;\n\t"
      "@ev add.s32 %1, %1, -32;\n\t"
      "cvt.u32.u64 x, %0;\n\t"
      "and.b32 x, x, 511;\n\t"
      "or.b32 x, x, %7;\n\t"
      "ld.shared.u8 %3, [x];\n\t"
      "and.b32 len, %3, 15;\n\t"
      "shr.b64 %0, %0, len;\n\t"
      "add.s32 %1, %1, len;\n\t"
      "cvt.u32.u64 x, %0;\n\t"
      "and.b32 x, x, 511;\n\t"
      "or.b32 x, x, %7;\n\t"
      "ld.shared.u8 %4, [x];\n\t"
      "and.b32 len, %4, 15;\n\t"
      "shr.b64 %0, %0, len;\n\t"
      "add.s32 %1, %1, len;\n\t"
      "}"
      : "+l"(buf), "+r"(nv), "+r"(off), "=&r"(e0), "=&r"(e1)
      : "r"(lt), "r"(base), "r"(lut), "r"(lenlut));
}


// Three symbols per ballot round: after a refill a lane holds at least 32 bits,
// so it cannot refill again within the next two symbols; each lane refills at
// most once in three consecutive symbols.  Its refill symbol k (level < 9 before
// symbol k, the earlier symbols' lengths from two chained length-only lookups
// of the current buffer) is known before any of the three is decoded; three
// cumulative ballots (refills at a slot <= 0, <= 1, <= 2; as in step_pair each
// follows from one comparison, nv + len_i + ... >= 0) order the refills as the
// format does (symbol i's refilling lanes in lane order, then i+1's, then
// i+2's), each lane's word index from one popc as in step_pair, and the word
// goes in right above the
// lane's valid bits before symbol i, at most 26 bits up (level < 9 + two codes
// of at most 9 bits), where the 64-bit buffer holds it; its multiplier
// 0x4000000 >> (nv + 18) is 1 << level for level <= 26.
__device__ __forceinline__ void step_triple(uint64_t &buf, int &nv, uint32_t &off, uint32_t base,
                                            uint32_t lut, uint32_t lenlut, unsigned lt,
                                            uint32_t &e0, uint32_t &e1, uint32_t &e2) {
  asm volatile(
      "{\n\t"
      ".reg .pred p0, q, ev;\n\t"
      ".reg .b32 x, lo, hi, l0, l1, t, b0, b1, b2, n1, mb, c, bs, a, w, m, len;\n\t"
      "setp.ge.s32 p0, %1, 0;\n\t"
      "mov.b64 {lo, hi}, %0;\n\t"
      "and.b32 x, lo, 511;\n\t"
      "or.b32 x, x, %9;\n\t"
      "ld.shared.u8 l0, [x];\n\t"
      "shf.r.clamp.b32 x, lo, hi, l0;\n\t"
      "and.b32 x, x, 511;\n\t"
      "or.b32 x, x, %9;\n\t"
      "ld.shared.u8 l1, [x];\n\t"
      "add.s32 t, %1, l0;\n\t"
      "setp.ge.s32 q, t, 0;\n\t"
      "add.s32 t, t, l1;\n\t"
      "setp.ge.s32 ev, t, 0;\n\t"
      "vote.sync.ballot.b32 b0, p0, 0xffffffff;\n\t"
      "vote.sync.ballot.b32 b1, q, 0xffffffff;\n\t"
      "vote.sync.ballot.b32 b2, ev, 0xffffffff;\n\t"
      "selp.b32 mb, b0, b1, q;\n\t"
      "selp.b32 mb, 0, mb, p0;\n\t"
      "selp.b32 bs, b1, b2, q;\n\t"
      "selp.b32 bs, b0, bs, p0;\n\t"
      "lop3.b32 mb, bs, mb, %6, 0xE4;\n\t"
      "popc.b32 c, mb;\n\t"
      "mad.lo.u32 a, c, 4, %2;\n\t"
      "and.b32 a, a, " XP_RING_MASK ";\n\t"
      "or.b32 a, a, %7;\n\t"
      "ld.shared.u32 w, [a];\n\t"
      "popc.b32 n1, b2;\n\t"
      "mad.lo.u32 %2, n1, 4, %2;\n\t"
      "add.s32 t, %1, 18;\n\t"
      "shr.b32 m, 67108864, t;\n\t"
      "@ev mad.wide.u32 %0, w, m, %0;\n\t"
      "@ev add.s32 %1, %1, -32;\n\t"
      "cvt.u32.u64 x, %0;\n\t"
      "and.b32 x, x, 511;\n\t"
      "or.b32 x, x, %8;\n\t"
      "ld.shared.u8 %3, [x];\n\t"
      "and.b32 len, %3, 15;\n\t"
      "shr.b64 %0, %0, len;\n\t"
      "add.s32 %1, %1, len;\n\t"
      "cvt.u32.u64 x, %0;\n\t"
      "and.b32 x, x, 511;\n\t"
      "or.b32 x, x, %8;\n\t"
      "ld.shared.u8 %4, [x];\n\t"
      "and.b32 len, %4, 15;\n\t"
      "shr.b64 %0, %0, len;\n\t"
      "add.s32 %1, %1, len;\n\t"
      "cvt.u32.u64 x, %0;\n\t"
      "and.b32 x, x, 511;\n\t"
      "or.b32 x, x, %8;\n\t"
      "ld.shared.u8 %5, [x];\n\t"
      "and.b32 len, %5, 15;\n\t"
      "shr.b64 %0, %0, len;\n\t"
      "add.s32 %1, %1, len;\n\t"
      "}"
      : "+l"(buf), "+r"(nv), "+r"(off), "=&r"(e0), "=&r"(e1), "=&r"(e2)
      : "r"(lt), "r"(base), "r"(lut), "r"(lenlut));
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

__global__ void __launch_bounds__(kWarps * 32, 10) decode_ring_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t s_dyn[];  // kWarps rings of 2 KiB, 2 KiB-aligned
  __shared__ __align__(512) uint8_t s_lut[kWarps][kLutBytes];
  __shared__ __align__(512) uint8_t s_len[kWarps][kLutBytes];  // lengths only
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
  // Three global round trips: the todo entry and the group's word range; the
  // skip list, cache/destination rows and LUT; then the group's first ring of
  // words.
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
  int nv = 8;  // 8 - level: level < 9 (a refill) iff nv >= 0
  uint32_t off = static_cast<uint32_t>(4 * (a_begin - a0));
  const uint32_t sl = static_cast<uint32_t>(__cvta_generic_to_shared(L));
  const uint32_t sn = static_cast<uint32_t>(__cvta_generic_to_shared(s_len[warp]));
  // Eight symbols in rounds of 3 + 3 + 2: their LUT entries summed at byte
  // offsets, symbols 0-3 into lo and 4-7 into hi.
  auto octet = [&](uint32_t &lo, uint32_t &hi) {
    uint32_t e[8];
    step_triple(buf, nv, off, base, sl, sn, lt, e[0], e[1], e[2]);
    step_triple(buf, nv, off, base, sl, sn, lt, e[3], e[4], e[5]);
    step_pair(buf, nv, off, base, sl, sn, lt, e[6], e[7]);
    lo = mad_u32(e[3], 1u << 24, mad_u32(e[2], 1u << 16, mad_u32(e[1], 1u << 8, e[0])));
    hi = mad_u32(e[7], 1u << 24, mad_u32(e[6], 1u << 16, mad_u32(e[5], 1u << 8, e[4])));
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
    if (pending && off + kMaxAdvance + kHalf >= filled) {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncwarp();
      pending = false;
    }
    uint32_t lohi[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t nw = h ? q1 : q0;
      uint32_t acc_lo, acc_hi;
      octet(acc_lo, acc_hi);
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
  dim3 grid(static_cast<unsigned>((groups + kWarps - 1) / kWarps), static_cast<unsigned>(K));
  decode_ring_kernel<<<grid, kWarps * 32, kRingSmem, as_stream(stream)>>>(a);
  return launch_status();
}
