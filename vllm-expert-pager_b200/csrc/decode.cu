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
// B200 mapping: one warp per group, several groups per CTA.
//  * The group's Huffman words arrive in refill order, so the warp holds a
//    96-word window in three registers per lane and hands each refilling lane
//    its word with two shuffles; the window slides by 32 words with one
//    coalesced load issued 32..64 words before its use.
//  * LUT lookups go to a 128-byte first-level table in shared memory: 32 words
//    in 32 distinct banks, so a warp's 32 random lookups never conflict.  Codes
//    longer than 7 bits (rare) fall back to the full 512-byte table.
//  * Nibble words are read coalesced (word m of all 32 lanes is contiguous).
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

__global__ void __launch_bounds__(kWarps * 32) decode_kernel(const __grid_constant__ DecodeArgs a) {
  __shared__ __align__(16) uint8_t s_lut[kWarps][kLutBytes];
  __shared__ __align__(16) uint8_t s_lut1[kWarps][128];
  const int64_t j = blockIdx.y;
  const int64_t e = a.todo[j];
  if (e < 0) return;
  if (a.skip)
    for (int64_t k = 0; k < a.K; ++k)
      if (a.skip[k] == e) return;
  if (a.cache_row[e] >= 0) return;  // copied raw from the cache slab
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t gg = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (gg >= a.n[0].G + a.n[1].G) return;
  const int which = gg < a.n[0].G ? 0 : 1;
  const DName &n = a.n[which];
  const int64_t g = which ? gg - a.n[0].G : gg;
  int64_t dst_row = a.dst_row[e];
  dst_row = dst_row > 0 ? dst_row : 0;

  // This row's LUT, and its conflict-free 7-bit first level (0 = longer code).
  uint8_t *L = s_lut[warp];
  uint8_t *L1 = s_lut1[warp];
  reinterpret_cast<uint4 *>(L)[lane] =
      reinterpret_cast<const uint4 *>(a.lut + (e * 2 + which) * kLutBytes)[lane];
  __syncwarp();
  for (int i = lane; i < 128; i += 32) {
    uint8_t v = L[i];
    L1[i] = (v & 15) <= 7 ? v : 0;
  }
  __syncwarp();

  const int64_t chunk = a.chunk, G = n.G;
  const uint8_t *rec = n.stg + j * n.P;
  const int64_t head = 4 * (G + 1);
  const int32_t *hdr = reinterpret_cast<const int32_t *>(rec);
  const uint32_t *nib = reinterpret_cast<const uint32_t *>(rec + head) + g * (chunk / 8) * 32;
  const uint32_t *huff = reinterpret_cast<const uint32_t *>(rec + head + n.N / 2);
  // Words of this group: [gstart[g], gstart[g+1]), never past the record.
  const int64_t maxw = (n.P - head - n.N / 2) / 4;
  const int64_t rend = hdr[g + 1] < maxw ? hdr[g + 1] : maxw;
  int64_t wbase = hdr[g];
  auto ld = [&](int64_t idx) -> uint32_t {
    return (idx >= 0 && idx < rend) ? __ldg(huff + idx) : 0u;
  };
  uint32_t w0 = ld(wbase + lane), w1 = ld(wbase + 32 + lane), w2 = ld(wbase + 64 + lane);
  uint64_t *out = reinterpret_cast<uint64_t *>(n.dst + dst_row * n.N + (g * 32 + lane) * chunk);

  uint64_t buf = 0;
  int level = 0, rel = 0;  // rel: next word of the group relative to wbase, < 32
  const unsigned lt = lanemask_lt();
  uint32_t nw_next = __ldg(nib + lane);
  for (int64_t m = 0; m < chunk / 8; ++m) {
    const uint32_t nw = nw_next;
    if (m + 1 < chunk / 8) nw_next = __ldg(nib + (m + 1) * 32 + lane);
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
      uint32_t ent = L1[buf & 127];
      if ((ent & 15) == 0) ent = L[buf & (kLutBytes - 1)];
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
    if (N <= 0 || N % (32 * chunk) || P % 4 || P < 4 * (N / (32 * chunk) + 1) + N / 2)
      return XP_EINVAL;
    if (!stgs[i] || !dsts[i] || !aligned(stgs[i], 4) || !aligned(dsts[i], 8)) return XP_EINVAL;
    a.n[i] = DName{static_cast<const uint8_t *>(stgs[i]), P, static_cast<uint8_t *>(dsts[i]), N,
                   N / (32 * chunk)};
  }
  const int64_t groups = a.n[0].G + a.n[1].G;
  dim3 grid(static_cast<unsigned>((groups + kWarps - 1) / kWarps), static_cast<unsigned>(K));
  decode_kernel<<<grid, kWarps * 32, 0, as_stream(stream)>>>(a);
  return launch_status();
}
