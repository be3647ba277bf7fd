// Host encoder of the fp8-exponent Huffman records (load time).
//
// Produces byte-identical records to monochromegane/vllm-expert-pager
// src/vllm_expert_pager/codec.py:125-193 (the record format of codec.py:22-26):
// the same length-limited Huffman construction (codec.py:61-87, including the
// heap's tie order), the same canonical bit-reversed codes (codec.py:90-114) and
// the same refill order of the words (codec.py:150-181).  The reference runs it
// as torch ops on the GPU at load time; here it is a plain loop over one row.
#include <stdint.h>
#include <string.h>

#include <vector>

#include "xpager.h"

namespace {

constexpr int kLimit = 9;
constexpr int kLanes = 32;

// Plain Huffman lengths.  The reference pushes (count, tiebreak, members) on a
// heap and pops the two smallest (count, tiebreak); leaves have tiebreak = the
// symbol, merged nodes take 16, 17, ... in creation order.
void huffman_lengths(const double *counts, int *lengths) {
  double c[32];
  int tie[32];
  uint32_t members[32];
  int live = 16, next = 16;
  for (int i = 0; i < 16; ++i) {
    c[i] = counts[i];
    tie[i] = i;
    members[i] = 1u << i;
    lengths[i] = 0;
  }
  auto less = [&](int a, int b) { return c[a] < c[b] || (c[a] == c[b] && tie[a] < tie[b]); };
  while (live > 1) {
    int a = 0;
    for (int i = 1; i < live; ++i)
      if (less(i, a)) a = i;
    // remove a
    double ca = c[a];
    uint32_t ma = members[a];
    c[a] = c[live - 1], tie[a] = tie[live - 1], members[a] = members[live - 1];
    --live;
    int b = 0;
    for (int i = 1; i < live; ++i)
      if (less(i, b)) b = i;
    double cb = c[b];
    uint32_t mb = members[b];
    c[b] = c[live - 1], tie[b] = tie[live - 1], members[b] = members[live - 1];
    --live;
    uint32_t m = ma | mb;
    for (int s = 0; s < 16; ++s)
      if (m >> s & 1) ++lengths[s];
    c[live] = ca + cb;
    tie[live] = next++;
    members[live] = m;
    ++live;
  }
}

// codec.py:76-87: raise rare counts until every length is <= LIMIT.
void code_lengths(const int64_t *hist, int *lengths) {
  double counts[16];
  for (int i = 0; i < 16; ++i) counts[i] = static_cast<double>(hist[i] > 1 ? hist[i] : 1);
  for (int k = 0;; ++k) {
    if (k > 0) {
      double sum = 0;
      for (int i = 0; i < 16; ++i) sum += counts[i];
      double floor_ = sum / static_cast<double>(1 << (kLimit - k));
      for (int i = 0; i < 16; ++i) counts[i] = counts[i] > floor_ ? counts[i] : floor_;
    }
    huffman_lengths(counts, lengths);
    int mx = 0;
    for (int i = 0; i < 16; ++i) mx = lengths[i] > mx ? lengths[i] : mx;
    if (mx <= kLimit) return;
  }
}

}  // namespace

extern "C" int xp_encode_row(const uint8_t *raw, int64_t n, int64_t pitch, int64_t chunk,
                             uint8_t *record, uint8_t *lut, int64_t *used) {
  if (!raw || !record || !lut || chunk <= 0 || chunk % 8 || n <= 0 || n % (chunk * kLanes))
    return XP_EINVAL;
  const int64_t C = n / chunk, G = n / (chunk * kLanes);

  int64_t hist[16] = {0};
  for (int64_t i = 0; i < n; ++i) ++hist[(raw[i] >> 3) & 15];
  int len[16];
  code_lengths(hist, len);
  // Canonical codes in (length, symbol) order, stored bit-reversed (codec.py:94-106).
  int order[16];
  for (int i = 0; i < 16; ++i) order[i] = i;
  for (int i = 1; i < 16; ++i)
    for (int j = i; j > 0 && (len[order[j]] < len[order[j - 1]] ||
                              (len[order[j]] == len[order[j - 1]] && order[j] < order[j - 1]));
         --j) {
      int t = order[j];
      order[j] = order[j - 1];
      order[j - 1] = t;
    }
  uint32_t canon[16], code[16];
  uint32_t cc = 0;
  for (int i = 0; i < 16; ++i) {
    int s = order[i];
    if (i) cc = (cc + 1) << (len[s] - len[order[i - 1]]);
    canon[s] = cc;
  }
  for (int s = 0; s < 16; ++s) {
    uint32_t r = 0;
    for (int b = 0; b < len[s]; ++b) r |= ((canon[s] >> b) & 1u) << (len[s] - 1 - b);
    code[s] = r;
  }
  // LUT (codec.py:107-114).
  int filled = 0;
  for (int s = 0; s < 16; ++s)
    for (uint32_t hi = 0; hi < (1u << (kLimit - len[s])); ++hi) {
      lut[code[s] | (hi << len[s])] = static_cast<uint8_t>((s << 4) | len[s]);
      ++filled;
    }
  if (filled != (1 << kLimit)) return XP_EINVAL;  // not a complete prefix code

  // Per chunk: bit positions, word count, and the symbol index of each refill:
  // the k-th refill is at the first symbol i with before[i] >= 32k - (LIMIT-1).
  std::vector<int64_t> nw(C), wbase(C);
  std::vector<int32_t> at;  // refill symbol index per (chunk, k), flattened by wbase
  int64_t total = 0;
  for (int64_t c = 0; c < C; ++c) {
    const uint8_t *v = raw + c * chunk;
    int64_t before = 0, last_before = 0;
    for (int64_t i = 0; i < chunk; ++i) {
      last_before = before;
      before += len[(v[i] >> 3) & 15];
    }
    nw[c] = (last_before + (kLimit - 1)) / 32 + 1;
    wbase[c] = total;
    total += nw[c];
  }
  const int64_t head = 4 * (G + 1) + n / 2;
  const int64_t nbytes = head + 4 * total;
  if (used) *used = nbytes;
  if (nbytes > pitch) return XP_EPITCH;

  std::vector<uint32_t> words(total + 1, 0);
  at.assign(total, 0);
  for (int64_t c = 0; c < C; ++c) {
    const uint8_t *v = raw + c * chunk;
    int64_t bit = wbase[c] * 32, before = 0, k = 0;
    for (int64_t i = 0; i < chunk; ++i) {
      while (k < nw[c] && before >= 32 * k - (kLimit - 1)) at[wbase[c] + k++] = static_cast<int32_t>(i);
      const int s = (v[i] >> 3) & 15;
      const uint64_t bits = static_cast<uint64_t>(code[s]) << ((bit + before) & 31);
      const int64_t w = (bit + before) >> 5;
      words[w] |= static_cast<uint32_t>(bits);
      words[w + 1] |= static_cast<uint32_t>(bits >> 32);
      before += len[s];
    }
  }

  memset(record, 0, static_cast<size_t>(pitch));
  // Header: gstart[G+1] (codec.py:182-187).
  int32_t *hdr = reinterpret_cast<int32_t *>(record);
  int64_t acc = 0;
  for (int64_t g = 0; g < G; ++g) {
    int32_t gs = static_cast<int32_t>(acc);
    memcpy(hdr + g, &gs, 4);
    for (int64_t l = 0; l < kLanes; ++l) acc += nw[g * kLanes + l];
  }
  {
    int32_t t = static_cast<int32_t>(acc);
    memcpy(hdr + G, &t, 4);
  }
  // Sign/mantissa nibbles in (group, word, lane) order (codec.py:140-143).
  uint8_t *fixed = record + 4 * (G + 1);
  const int64_t M = chunk / 8;
  for (int64_t g = 0; g < G; ++g)
    for (int64_t l = 0; l < kLanes; ++l) {
      const uint8_t *v = raw + (g * kLanes + l) * chunk;
      for (int64_t m = 0; m < M; ++m)
        for (int b = 0; b < 4; ++b) {
          uint8_t x0 = v[8 * m + 2 * b], x1 = v[8 * m + 2 * b + 1];
          uint8_t s0 = static_cast<uint8_t>(((x0 >> 7) << 3) | (x0 & 7));
          uint8_t s1 = static_cast<uint8_t>(((x1 >> 7) << 3) | (x1 & 7));
          fixed[((g * M + m) * kLanes + l) * 4 + b] = static_cast<uint8_t>(s0 | (s1 << 4));
        }
    }
  // Huffman words per group in (refill symbol index, lane) order: a 32-way
  // merge of the lanes' refill lists (codec.py:177-181).
  uint8_t *out = record + head;
  int64_t pos = 0;
  for (int64_t g = 0; g < G; ++g) {
    int64_t next[kLanes] = {0};
    for (int64_t i = 0; i < chunk; ++i)
      for (int64_t l = 0; l < kLanes; ++l) {
        const int64_t c = g * kLanes + l;
        while (next[l] < nw[c] && at[wbase[c] + next[l]] == i) {
          memcpy(out + 4 * pos++, &words[wbase[c] + next[l]], 4);
          ++next[l];
        }
      }
  }
  return pos == total ? XP_OK : XP_EINVAL;
}
