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
//  * Several symbols per ballot round (round3, round2; 8 symbols in rounds of
//    3 + 3 + 2): a lane refills at most once in three consecutive symbols, its
//    refill symbol follows from table lookups in its current buffer, and its
//    word can be inserted above its valid bits before the round's first
//    symbol; so one round of ballots and one word load serves two or three
//    symbols.  Only the lanes whose refill came at or before one of the
//    round's first two symbols look that symbol up again (predicated loads).
//  * Position-based symbol chain: a per-warp table of 16-bit entries
//    len | sym << 12 whose low five bits are the code length, the stream kept
//    one bit up in a 64-bit register pair so a window's table address is one
//    AND/OR; each next window is one wrapping funnel shift by the previous
//    entry, and the buffer is shifted once per round by the sum of the
//    round's entries.  Per symbol: address, load, funnel shift.
//  * The level counter sits in the top seven bits of a register, so every
//    length update is an entry x 2^25 multiply-add on the FMA pipe; the
//    exponent fields are packed by multiplies too, and the sign/mantissa
//    nibbles spread by multiplies and one byte permute.  The integer ALU pipe
//    (one warp instruction per two cycles per scheduler) takes the rest.
//  * Each lane stores 32 bytes per 32 symbols (16 per 16 where rows are not
//    32-byte aligned); nibble words are loaded 32 symbols ahead.
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
                                    const uint16_t *T, int lane) {
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
      const uint32_t ent = T[buf & (kLutBytes - 1)];  // len | sym << 12
      const uint32_t len = ent & 15;
      buf >>= len;
      level -= static_cast<int>(len);
      const uint32_t s = (nw >> (4 * k)) & 15;
      const uint32_t byte = ((s & 8) << 4) | ((ent >> 12) << 3) | (s & 7);
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
__device__ __forceinline__ uint32_t mulhi_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.hi.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t madhi_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("mad.hi.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// Bitwise select: (a & m) | (b & ~m), one three-input logic op.
__device__ __forceinline__ uint32_t bitsel(uint32_t a, uint32_t b, uint32_t m) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(d) : "r"(a), "r"(b), "r"(m));
  return d;
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
#define XP_RING_MASK "2047"  // kRing - 1, spelled for the round functions' PTX
static_assert(kRing == 2048, "XP_RING_MASK spells kRing - 1");
// Most stream bytes a valid record's refills consume in 16 symbols: a lane
// refills at most once every 3 symbols, so 6 words per lane.
constexpr uint32_t kMaxAdvance = 6 * 32 * 4;
// Dynamic shared memory per CTA: kWarps rings plus the slack that aligns them.
constexpr size_t kRingSmem = kWarps * kRing + kRing;

// Decode table: per warp, 512 16-bit entries len | sym << 12 built from the
// row's 512-byte LUT (sym << 4 | len), the entry of window w at byte 2w of a
// 1 KiB-aligned block.  Bit buffer: the lane's stream bits sit one bit up in a
// 64-bit register pair lo, hi (stream bit j at bit j + 1), so a window's table
// address is one AND/OR of the register holding it ((x & mask) | table, the
// mask keeping as many window bits as the row's longest code).
// An entry's low five bits are its code length (bits 5-11 are zero), which is
// all a wrapping funnel shift reads of its shift amount: the next window is
// shf.r.wrap(lo, hi, entry), the sum of a round's entries shifts the buffer,
// and the symbol bits above never matter.
//
// Level counter: nv = (26 - level) << 25 (the lane's valid bit count in the
// top seven bits).  A lane refills before a symbol iff level < 9 there, i.e.
// nv + (lengths of the round's earlier symbols) << 25 >= 18 << 25; an entry
// times 2^25 is exactly its length << 25 (the symbol bits leave the register),
// so every level update is one multiply-add on the FMA pipe.  A refilling
// lane inserts its word w as lo += low(w * 2^(level + 1)), hi += high(...),
// two multiply-adds that carry nowhere (the bits above the valid ones are
// zero); 2^(level + 1) = 2^27 >> (nv >> 25).
constexpr int kNvStart = 26 << 25;  // level 0

// Three symbols per ballot round: after a refill a lane holds at least 32 bits,
// so it cannot refill again within the next two symbols; each lane refills at
// most once in three consecutive symbols.  Its refill symbol k (level < 9 before
// symbol k) is known before the word arrives: the round's first two entries are
// looked up in the current buffer, exact for every symbol before a lane's
// refill symbol (>= 9 valid bits there).  Three cumulative ballots (refill at a
// slot <= 0, <= 1, <= 2) order the refills as the format does (symbol i's
// refilling lanes in lane order, then i+1's, then i+2's); a lane's word index
// is popc(B_{k-1} | (B_k & lanes below it)), one shared load gives each
// refilling lane its word (the others keep a zero word, so the insert itself
// needs no predicate), and the word goes in right above the lane's valid
// bits before symbol i (at most bit 27 with the one-bit offset: level < 9 + two
// codes of at most 9 bits), where the 64-bit buffer holds it.  Then the
// symbols are decoded from the new buffer; the first two are looked up again
// only by the lanes whose refill came at or before them (predicated loads: the
// other lanes' entries from the current buffer are already exact), the third
// by every lane.  Returns the three table entries.
__device__ __forceinline__ void round3(uint32_t &blo, uint32_t &bhi, int &nv, uint32_t &off,
                                       uint32_t ring, uint32_t tab, uint32_t msk, unsigned lt,
                                       uint32_t &e0,
                                       uint32_t &e1, uint32_t &e2) {
  const uint32_t k25 = 1u << 25;
  asm volatile(
      "{\n\t"
      ".reg .pred p0, q, ev;\n\t"
      ".reg .b32 lo, hi, x, a, t1, t2, b0, b1, b2, mb, bs, c, n2, w, m, s, z;\n\t"
      "mov.b32 z, 0;\n\t"
      "mov.b32 w, 0;\n\t"
      "mov.b32 lo, %0;\n\t"
      "mov.b32 hi, %1;\n\t"
      "and.b32 a, lo, %11;\n\t"
      "or.b32 a, a, %8;\n\t"
      "ld.shared.u16 %4, [a];\n\t"
      "shf.r.wrap.b32 x, lo, hi, %4;\n\t"
      "and.b32 a, x, %11;\n\t"
      "or.b32 a, a, %8;\n\t"
      "ld.shared.u16 %5, [a];\n\t"
      "mad.lo.u32 t1, %4, %10, %2;\n\t"
      "mad.lo.u32 t2, %5, %10, t1;\n\t"
      "setp.ge.s32 p0, %2, 603979776;\n\t"
      "setp.ge.s32 q, t1, 603979776;\n\t"
      "setp.ge.s32 ev, t2, 603979776;\n\t"
      "vote.sync.ballot.b32 b0, p0, 0xffffffff;\n\t"
      "vote.sync.ballot.b32 b1, q, 0xffffffff;\n\t"
      "vote.sync.ballot.b32 b2, ev, 0xffffffff;\n\t"
      "selp.b32 bs, b1, b2, q;\n\t"
      "selp.b32 bs, b0, bs, p0;\n\t"
      "selp.b32 mb, b0, b1, q;\n\t"
      "selp.b32 mb, 0, mb, p0;\n\t"
      "lop3.b32 mb, bs, mb, %9, 0xE4;\n\t"
      "popc.b32 c, mb;\n\t"
      "mad.lo.u32 a, c, 4, %3;\n\t"
      "and.b32 a, a, " XP_RING_MASK ";\n\t"
      "or.b32 a, a, %7;\n\t"
      "@ev ld.shared.u32 w, [a];\n\t"
      "popc.b32 n2, b2;\n\t"
      "mad.lo.u32 %3, n2, 4, %3;\n\t"
      "shr.u32 s, %2, 25;\n\t"
      "shr.b32 m, 134217728, s;\n\t"
      "mad.lo.u32 lo, w, m, lo;\n\t"
      "mad.hi.u32 hi, w, m, hi;\n\t"
      "@ev add.s32 %2, %2, -1073741824;\n\t"
      "and.b32 a, lo, %11;\n\t"
      "or.b32 a, a, %8;\n\t"
      "@p0 ld.shared.u16 %4, [a];\n\t"
      "shf.r.wrap.b32 x, lo, hi, %4;\n\t"
      "and.b32 a, x, %11;\n\t"
      "or.b32 a, a, %8;\n\t"
      "@q ld.shared.u16 %5, [a];\n\t"
      "shf.r.wrap.b32 x, x, z, %5;\n\t"
      "and.b32 a, x, %11;\n\t"
      "or.b32 a, a, %8;\n\t"
      "ld.shared.u16 %6, [a];\n\t"
      "add.s32 s, %4, %5;\n\t"
      "add.s32 s, s, %6;\n\t"
      "shf.r.wrap.b32 x, lo, hi, s;\n\t"
      "shf.r.wrap.b32 hi, hi, z, s;\n\t"
      "mov.b32 %0, x;\n\t"
      "mov.b32 %1, hi;\n\t"
      "mad.lo.u32 %2, s, %10, %2;\n\t"
      "}"
      : "+r"(blo), "+r"(bhi), "+r"(nv), "+r"(off), "=&r"(e0), "=&r"(e1), "=&r"(e2)
      : "r"(ring), "r"(tab), "r"(lt), "r"(k25), "r"(msk));
}

// Two symbols per ballot round, as round3 with one look-ahead entry: a lane
// refills at symbol i (level < 9) or at i+1 (level - len_i < 9), and the
// word goes in at most at bit 18.  Returns the two table entries.
__device__ __forceinline__ void round2(uint32_t &blo, uint32_t &bhi, int &nv, uint32_t &off,
                                       uint32_t ring, uint32_t tab, uint32_t msk, unsigned lt,
                                       uint32_t &e0,
                                       uint32_t &e1) {
  const uint32_t k25 = 1u << 25;
  asm volatile(
      "{\n\t"
      ".reg .pred p0, ev;\n\t"
      ".reg .b32 lo, hi, x, a, t1, b0, b1, mb, bs, c, n1, w, m, s, z;\n\t"
      "mov.b32 z, 0;\n\t"
      "mov.b32 w, 0;\n\t"
      "mov.b32 lo, %0;\n\t"
      "mov.b32 hi, %1;\n\t"
      "and.b32 a, lo, %10;\n\t"
      "or.b32 a, a, %7;\n\t"
      "ld.shared.u16 %4, [a];\n\t"
      "mad.lo.u32 t1, %4, %9, %2;\n\t"
      "setp.ge.s32 p0, %2, 603979776;\n\t"
      "setp.ge.s32 ev, t1, 603979776;\n\t"
      "vote.sync.ballot.b32 b0, p0, 0xffffffff;\n\t"
      "vote.sync.ballot.b32 b1, ev, 0xffffffff;\n\t"
      "selp.b32 mb, 0, b0, p0;\n\t"
      "selp.b32 bs, b0, b1, p0;\n\t"
      "lop3.b32 mb, bs, mb, %8, 0xE4;\n\t"
      "popc.b32 c, mb;\n\t"
      "mad.lo.u32 a, c, 4, %3;\n\t"
      "and.b32 a, a, " XP_RING_MASK ";\n\t"
      "or.b32 a, a, %6;\n\t"
      "@ev ld.shared.u32 w, [a];\n\t"
      "popc.b32 n1, b1;\n\t"
      "mad.lo.u32 %3, n1, 4, %3;\n\t"
      "shr.u32 s, %2, 25;\n\t"
      "shr.b32 m, 134217728, s;\n\t"
      "mad.lo.u32 lo, w, m, lo;\n\t"
      "mad.hi.u32 hi, w, m, hi;\n\t"
      "@ev add.s32 %2, %2, -1073741824;\n\t"
      "and.b32 a, lo, %10;\n\t"
      "or.b32 a, a, %7;\n\t"
      "@p0 ld.shared.u16 %4, [a];\n\t"
      "shf.r.wrap.b32 x, lo, hi, %4;\n\t"
      "and.b32 a, x, %10;\n\t"
      "or.b32 a, a, %7;\n\t"
      "ld.shared.u16 %5, [a];\n\t"
      "add.s32 s, %4, %5;\n\t"
      "shf.r.wrap.b32 x, lo, hi, s;\n\t"
      "shf.r.wrap.b32 hi, hi, z, s;\n\t"
      "mov.b32 %0, x;\n\t"
      "mov.b32 %1, hi;\n\t"
      "mad.lo.u32 %2, s, %9, %2;\n\t"
      "}"
      : "+r"(blo), "+r"(bhi), "+r"(nv), "+r"(off), "=&r"(e0), "=&r"(e1)
      : "r"(ring), "r"(tab), "r"(lt), "r"(k25), "r"(msk));
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

// V8: the output goes out as one 32-byte store per lane per 32 symbols (rows
// 32-byte aligned and chunk a multiple of 32), else one 16-byte store per 16
// symbols.  Each lane's stores land 512 bytes (its chunk) from its neighbours',
// so a warp's store touches 32 lines whatever its width; twice the bytes per
// store halves the store traffic through the L1 data pipe, which this kernel
// shares with its table lookups.
template <bool V8>
__global__ void __launch_bounds__(kWarps * 32, 10) decode_ring_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t s_dyn[];  // kWarps rings of 2 KiB, 2 KiB-aligned
  __shared__ __align__(1024) uint16_t s_tab[kWarps][kLutBytes];  // len | sym << 12
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
  // The decode table: LUT byte sym << 4 | len -> 16-bit len | sym << 12, each
  // lane converting its 16 bytes (two per 32-bit word).
  uint16_t *T = s_tab[warp];
  {
    const uint32_t v[4] = {lut_v.x, lut_v.y, lut_v.z, lut_v.w};
    uint32_t t[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = __byte_perm(v[i / 2], 0, (i & 1) ? 0x4342 : 0x4140);  // bytes -> halves
      t[i] = (b & 0x000F000Fu) | ((b & 0x00F000F0u) << 8);
    }
    reinterpret_cast<uint4 *>(T)[2 * lane] = make_uint4(t[0], t[1], t[2], t[3]);
    reinterpret_cast<uint4 *>(T)[2 * lane + 1] = make_uint4(t[4], t[5], t[6], t[7]);
  }
  // Windows are looked up with as many bits as the row's longest code: the
  // LUT repeats above that length, so entries [0, 2^maxlen) hold every code,
  // and fewer distinct table words mean fewer shared-memory bank conflicts.
  uint32_t msk;
  {
    const uint32_t m4 = __vmaxu4(__vmaxu4(lut_v.x & 0x0F0F0F0Fu, lut_v.y & 0x0F0F0F0Fu),
                                 __vmaxu4(lut_v.z & 0x0F0F0F0Fu, lut_v.w & 0x0F0F0F0Fu));
    uint32_t mx = max(max(m4 & 255, (m4 >> 8) & 255), max((m4 >> 16) & 255, m4 >> 24));
    mx = __reduce_max_sync(kFull, mx);
    mx = mx < 1 ? 1 : (mx > kLimit ? kLimit : mx);
    msk = ((1u << mx) - 1) << 1;  // table byte offsets 2w of the used windows w
  }
  dst_row = dst_row > 0 ? dst_row : 0;
  const uint32_t *nib = reinterpret_cast<const uint32_t *>(rec + head) + g * (chunk / 8) * 32;
  uint8_t *out_row = n.dst + dst_row * n.N + (g * 32 + lane) * chunk;
  const int64_t a_begin = huff_w + w_begin, a_end = huff_w + w_end;
  const int64_t a0 = a_begin & ~int64_t(3);  // 16-byte aligned (records are 16-byte aligned)
  if ((chunk / 8) % 2) {
    __syncwarp();
    decode_group_window(reinterpret_cast<const uint32_t *>(rec) + huff_w, w_begin, w_end, nib,
                        out_row, chunk, T, lane);
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
  uint32_t blo = 0, bhi = 0;
  int nv = kNvStart;
  uint32_t off = static_cast<uint32_t>(4 * (a_begin - a0));
  const uint32_t tab = static_cast<uint32_t>(__cvta_generic_to_shared(T));
  // Exponent fields of 4 symbols from their table entries len | sym << 12:
  // sym << (8k + 3) for symbol k, by e >> 9, e >> 1, e << 7, e << 15 as
  // multiplies.  The length bits those leave behind (len >> 1 at bits 0-2,
  // len << 7 at bits 7-10, len << 15 at bits 15-18) share no bit with the
  // exponent fields (bits 3-6 of each byte) or with one another, so the sum
  // carries nowhere and the caller keeps bits 3-6 of each byte.
  auto pack4 = [&](uint32_t e0, uint32_t e1, uint32_t e2, uint32_t e3) {
    return mad_u32(e3, 1u << 15, mad_u32(e2, 1u << 7, madhi_u32(e1, 1u << 31, mulhi_u32(e0, 1u << 23))));
  };
  // Eight symbols in rounds of 3 + 3 + 2 -> two output words: nibble word nw
  // holds the 8 sign/mantissa nibbles (symbol k at bits 4k..4k+3).  Nibbles
  // 0, 2, 4, 6 and 1, 3, 5, 7 go to the low halves of the bytes of two words,
  // times 17 copies each to its byte's high half, a byte permute interleaves
  // them in symbol order, and one select keeps the sign (bit 7) and mantissa
  // (bits 0-2) from there and the exponent (bits 3-6) from the entries.
  auto octet = [&](uint32_t nw, uint32_t &lo, uint32_t &hi) {
    uint32_t e[8];
    round3(blo, bhi, nv, off, base, tab, msk, lt, e[0], e[1], e[2]);
    round3(blo, bhi, nv, off, base, tab, msk, lt, e[3], e[4], e[5]);
    round2(blo, bhi, nv, off, base, tab, msk, lt, e[6], e[7]);
    const uint32_t ev = mul_u32(nw & 0x0F0F0F0Fu, 17u);
    const uint32_t od = mul_u32(mulhi_u32(nw, 1u << 28) & 0x0F0F0F0Fu, 17u);
    lo = bitsel(pack4(e[0], e[1], e[2], e[3]), __byte_perm(ev, od, 0x5140), 0x78787878u);
    hi = bitsel(pack4(e[4], e[5], e[6], e[7]), __byte_perm(ev, od, 0x7362), 0x78787878u);
  };
  const int steps = static_cast<int>(chunk / 8);
  // Nibble words of 8-value block k: np[32 k]; q0..q3 hold blocks m..m+3.
  const uint32_t *np = nib + lane;
  uint32_t q0 = __ldg(np);
  uint32_t q1 = __ldg(np + 32);
  uint32_t q2 = 0, q3 = 0;
  if (steps > 2) {
    q2 = __ldg(np + 64);
    q3 = __ldg(np + 96);
  }
  // Ring upkeep at the top of every 16 symbols, warp-uniform (off and filled
  // are the same in every lane).
  auto upkeep = [&]() {
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
  };
  // Sixteen symbols: two octets from the nibble words q0, q1; then the nibble
  // words move up and the next two are loaded (two iterations ahead; none past
  // the group's last block, steps being even).
  auto sixteen = [&](int m, uint32_t *w) {
    upkeep();
    octet(q0, w[0], w[1]);
    octet(q1, w[2], w[3]);
    q0 = q2;
    q1 = q3;
    np += 64;
    if (m + 4 < steps) {
      q2 = __ldg(np + 64);
      q3 = __ldg(np + 96);
    }
  };
  if (V8) {
    for (int m = 0; m < steps; m += 4) {
      uint32_t w[8];
      sixteen(m, w);
      sixteen(m + 2, w + 4);
      asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(out_row + 8 * m),
                   "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]),
                   "r"(w[7])
                   : "memory");
    }
  } else {
    uint4 *out = reinterpret_cast<uint4 *>(out_row);
#pragma unroll 2
    for (int m = 0; m < steps; m += 2) {
      uint32_t w[4];
      sixteen(m, w);
      out[m / 2] = make_uint4(w[0], w[1], w[2], w[3]);
    }
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
  if (K < 0 || K > 65535 || chunk < 8 || chunk % 8 || chunk > (int64_t(1) << 30)) return XP_EINVAL;
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
  // 32-byte stores when every lane chunk starts on a 32-byte boundary and
  // holds a whole number of 32-symbol blocks.
  const bool v8 = chunk % 32 == 0 && aligned(dst0, 32) && aligned(dst1, 32);
  if (v8)
    decode_ring_kernel<true><<<grid, kWarps * 32, kRingSmem, as_stream(stream)>>>(a);
  else
    decode_ring_kernel<false><<<grid, kWarps * 32, kRingSmem, as_stream(stream)>>>(a);
  return launch_status();
}
