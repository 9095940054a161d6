/*
 * rans_oracle.c -- TEST INFRASTRUCTURE ONLY: a plain-C restatement of the "VQ2A" interleaved
 * rANS byte-stream format that compressai_b200 uses for ANS-coded expert indices. The product
 * encoder (host) and decoder (GPU) live in compressai_b200/csrc/rans.cu; this file shares no
 * code with them and is used only by tests/ as the checker.
 *
 * Why a format of this repository: the reference entropy-codes indices with the third-party
 * `constriction` package (vq2/export.py:26-36, AnsCoder + Categorical), which is not installed
 * here and whose stream format no reference test pins, so parity with it is unpinned; the
 * reference's paged container stores raw indices (vq2/pack_35b_to_vq2m.py:143-147).
 *
 * Format (little-endian):
 *   off 0    u32 magic 0x41325156 ("VQ2A")
 *   off 4    u32 n_symbols (bytes)
 *   off 8    u32 n_chunks = ceil(n_symbols / 8192)
 *   off 12   u32 0
 *   off 16   u16 freq[2][256]   context 0 = even symbol positions, 1 = odd; each row sums to 4096
 *   off 1040 u32 chunk_off[n_chunks + 1]  (from stream start; the last = total size)
 *   chunks at chunk_off[c] (16-byte aligned): u32 state[64], u16 nwords[64], then the u16 words
 *   of stream 0, stream 1, ... each in decode order; padded with zeros to 16 bytes.
 * Chunk c holds symbols [8192c, 8192c + cnt); stream w codes chunk symbols w, w+64, w+128, ...
 * (all of one parity, so one context per stream). rANS: 32-bit state, L = 2^16, 16-bit words,
 * 12-bit scale. Encode (reverse order, from x = L): if x >= f << 20 emit x & 0xffff, x >>= 16;
 * x = ((x / f) << 12) + x % f + c. Decode: s = sym(x & 4095); x = f * (x >> 12) + (x & 4095) - c;
 * if x < L: x = (x << 16) | next word. A step takes at most one word, so a stream holds at most
 * as many words as symbols; a valid stream ends at x = L with every word consumed.
 * Frequencies: f[s] = 1 + floor(count[s] * 3840 / total); the remaining 4096 - sum(f) go, one
 * each, to the symbols with the largest (count[s] * 3840) % total, ties to the smaller symbol;
 * an empty context gets f = 16 everywhere.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MAGIC 0x41325156u
#define CH 8192
#define WAYS 64
#define CHDR (WAYS * 6)
#define SCALE 12
#define TOT 4096u
#define RL 65536u
#define HDR 1040

static void wr32(uint8_t* p, uint32_t v) { p[0] = v; p[1] = v >> 8; p[2] = v >> 16; p[3] = v >> 24; }
static uint32_t rd32(const uint8_t* p) { return p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24); }
static void wr16(uint8_t* p, uint16_t v) { p[0] = v; p[1] = v >> 8; }
static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

void oracle_quantize(const uint64_t* count, uint16_t* freq) {
  uint64_t total = 0;
  for (int s = 0; s < 256; ++s) total += count[s];
  if (total == 0) {
    for (int s = 0; s < 256; ++s) freq[s] = 16;
    return;
  }
  uint64_t rem[256];
  uint32_t sum = 0;
  for (int s = 0; s < 256; ++s) {
    uint64_t q = count[s] * 3840u;
    freq[s] = (uint16_t)(1 + q / total);
    rem[s] = q % total;
    sum += freq[s];
  }
  uint32_t left = TOT - sum;
  /* repeatedly pick the largest remainder (smallest symbol on ties) */
  char used[256] = {0};
  for (uint32_t k = 0; k < left; ++k) {
    int best = -1;
    for (int s = 0; s < 256; ++s)
      if (!used[s] && (best < 0 || rem[s] > rem[best])) best = s;
    used[best] = 1;
    freq[best] += 1;
  }
}

int64_t oracle_bound(int64_t n) {
  int64_t nc = (n + CH - 1) / CH;
  int64_t hdr = (HDR + 4 * (nc + 1) + 15) / 16 * 16;
  /* per chunk: states and counts + at most one word per symbol + pad */
  return hdr + nc * (CHDR + 2 * CH + 16);
}

static int64_t stream_symbols(int64_t cntc, int w) { return cntc > w ? (cntc - w + WAYS - 1) / WAYS : 0; }

int64_t oracle_encode(const uint8_t* sym, int64_t n, uint8_t* out, int64_t cap) {
  if (n < 0 || n > 0x7fffffff || cap < oracle_bound(n)) return -1;
  memset(out, 0, (size_t)cap);
  uint64_t cnt[2][256];
  memset(cnt, 0, sizeof cnt);
  for (int64_t i = 0; i < n; ++i) cnt[i & 1][sym[i]]++;
  uint16_t f[2][256];
  uint32_t c[2][256];
  for (int k = 0; k < 2; ++k) {
    oracle_quantize(cnt[k], f[k]);
    uint32_t a = 0;
    for (int s = 0; s < 256; ++s) { c[k][s] = a; a += f[k][s]; }
  }
  int64_t nc = (n + CH - 1) / CH;
  wr32(out, MAGIC);
  wr32(out + 4, (uint32_t)n);
  wr32(out + 8, (uint32_t)nc);
  wr32(out + 12, 0);
  for (int k = 0; k < 2; ++k)
    for (int s = 0; s < 256; ++s) wr16(out + 16 + 2 * (k * 256 + s), f[k][s]);
  int64_t pos = (HDR + 4 * (nc + 1) + 15) / 16 * 16;
  uint16_t tmp[CH / WAYS + 4];
  for (int64_t ch = 0; ch < nc; ++ch) {
    wr32(out + HDR + 4 * ch, (uint32_t)pos);
    int64_t base = ch * CH;
    int64_t cntc = n - base < CH ? n - base : CH;
    uint8_t* hdr = out + pos;
    int64_t wpos = pos + CHDR;
    for (int w = 0; w < WAYS; ++w) {
      int k = w & 1;
      uint32_t x = RL;
      int nw = 0;
      for (int64_t j = stream_symbols(cntc, w) - 1; j >= 0; --j) {
        uint8_t s = sym[base + w + j * WAYS];
        uint32_t fs = f[k][s];
        if (x >= (fs << 20)) { tmp[nw++] = (uint16_t)(x & 0xffff); x >>= 16; }
        x = ((x / fs) << SCALE) + (x % fs) + c[k][s];
      }
      wr32(hdr + 4 * w, x);
      wr16(hdr + 4 * WAYS + 2 * w, (uint16_t)nw);
      for (int j = nw - 1; j >= 0; --j) { wr16(out + wpos, tmp[j]); wpos += 2; }
    }
    pos = (wpos + 15) / 16 * 16;
  }
  wr32(out + HDR + 4 * nc, (uint32_t)pos);
  return pos;
}

/* returns 0 on success, a nonzero code for a malformed stream */
int oracle_decode(const uint8_t* in, int64_t nbytes, uint8_t* out, int64_t out_cap) {
  if (nbytes < HDR + 4 || rd32(in) != MAGIC) return 1;
  int64_t n = rd32(in + 4), nc = rd32(in + 8);
  if (nc != (n + CH - 1) / CH || n > out_cap || HDR + 4 * (nc + 1) > nbytes) return 2;
  uint16_t f[2][256];
  uint32_t c[2][256];
  uint8_t s2[2][TOT];
  for (int k = 0; k < 2; ++k) {
    uint32_t a = 0;
    for (int s = 0; s < 256; ++s) {
      f[k][s] = rd16(in + 16 + 2 * (k * 256 + s));
      if (f[k][s] == 0) return 3;
      c[k][s] = a;
      for (uint32_t q = 0; q < f[k][s] && a + q < TOT; ++q) s2[k][a + q] = (uint8_t)s;
      a += f[k][s];
    }
    if (a != TOT) return 3;
  }
  for (int64_t ch = 0; ch < nc; ++ch) {
    int64_t o0 = rd32(in + HDR + 4 * ch), o1 = rd32(in + HDR + 4 * (ch + 1));
    if (o0 < (HDR + 4 * (nc + 1) + 15) / 16 * 16 || o0 + CHDR > o1 || o1 > nbytes) return 4;
    int64_t base = ch * CH, cntc = n - base < CH ? n - base : CH;
    int64_t wp = o0 + CHDR, all = 0;
    for (int w = 0; w < WAYS; ++w) { /* word counts: per stream <= symbols, all inside the chunk */
      int64_t nw = rd16(in + o0 + 4 * WAYS + 2 * w);
      if (nw > stream_symbols(cntc, w)) return 5;
      all += nw;
    }
    if (wp + 2 * all > o1) return 5;
    for (int w = 0; w < WAYS; ++w) {
      int k = w & 1;
      uint32_t x = rd32(in + o0 + 4 * w);
      int64_t nw = rd16(in + o0 + 4 * WAYS + 2 * w);
      int64_t wend = wp + 2 * nw;
      for (int64_t i = w; i < cntc; i += WAYS) {
        uint32_t slot = x & (TOT - 1);
        uint8_t s = s2[k][slot];
        x = f[k][s] * (x >> SCALE) + slot - c[k][s];
        if (x < RL) {
          if (wp >= wend) return 6;
          x = (x << 16) | rd16(in + wp);
          wp += 2;
        }
        out[base + i] = s;
      }
      if (x != RL || wp != wend) return 7;
    }
  }
  return 0;
}
