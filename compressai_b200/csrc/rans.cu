// Interleaved rANS coding of index byte streams ("VQ2A" format): host encoder and GPU decoder.
//
// ANS-coded expert containers store each expert's gate_up / down index tensors as one stream
// each; a paged miss copies the compressed record to the device and this decoder expands it
// straight into the slot. Format (little-endian; also stated in include/vq2_b200.h):
//   header: u32 magic "VQ2A", u32 n_symbols, u32 n_chunks = ceil(n / 8192), u32 0,
//           u16 freq[2][256] (context = symbol position parity; rows sum to 4096),
//           u32 chunk_off[n_chunks + 1] (the last is the total size), zero pad to 16 bytes;
//   chunk:  u32 state[64], u16 nwords[64], u16 words of stream 0, stream 1, ... (decode order),
//           zero pad to 16 bytes. Stream w codes chunk symbols w, w+64, w+128, ...
// rANS: 32-bit state, lower bound L = 2^16, 16-bit renormalisation words, 12-bit scale.
// The reference codes indices with the third-party `constriction` ANS coder
// (vq2/export.py:26-36), which is not available here; this is a format of this repository.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <vector>

#include "gemv.cuh"

namespace vq2 {

constexpr uint32_t kAnsMagic = 0x41325156u;  // "VQ2A"
constexpr int kAnsChunk = 8192;
constexpr int kAnsWays = 64;                   // rANS streams per chunk
constexpr int kAnsChunkHdr = kAnsWays * 6;     // states (u32) + word counts (u16)
constexpr int kAnsScale = 12;
constexpr uint32_t kAnsTotal = 1u << kAnsScale;
constexpr uint32_t kAnsLow = 1u << 16;
constexpr int kAnsHeader = 16 + 2 * 2 * 256;  // 1040: fields + frequency tables

__host__ __device__ inline int64_t ans_header_bytes(int64_t nc) { return (kAnsHeader + 4 * (nc + 1) + 15) / 16 * 16; }

// Symbols of stream w in a chunk of cnt symbols.
__host__ __device__ inline int ans_stream_symbols(int cnt, int w) { return cnt > w ? (cnt - w + kAnsWays - 1) / kAnsWays : 0; }

int64_t ans_bound(int64_t n) {
  const int64_t nc = (n + kAnsChunk - 1) / kAnsChunk;
  return ans_header_bytes(nc) + nc * (kAnsChunkHdr + 2 * kAnsChunk + 16);
}

// Quantized frequencies summing to 4096, every symbol >= 1: 1 + floor(count * 3840 / total),
// the leftover units to the largest remainders (count * 3840 mod total), ties to smaller symbols.
static void ans_quantize(const uint64_t* count, uint16_t* freq) {
  uint64_t total = 0;
  for (int s = 0; s < 256; ++s) total += count[s];
  if (total == 0) {
    std::fill(freq, freq + 256, uint16_t(16));
    return;
  }
  std::vector<std::pair<uint64_t, int>> order;  // (remainder, symbol)
  uint32_t used = 0;
  for (int s = 0; s < 256; ++s) {
    const uint64_t q = count[s] * 3840u;
    freq[s] = static_cast<uint16_t>(1 + q / total);
    used += freq[s];
    order.emplace_back(q % total, s);
  }
  std::stable_sort(order.begin(), order.end(),
                   [](const std::pair<uint64_t, int>& a, const std::pair<uint64_t, int>& b) {
                     return a.first > b.first;  // stable: equal remainders keep ascending symbols
                   });
  for (uint32_t k = 0; k < kAnsTotal - used; ++k) freq[order[k].second] += 1;
}

static inline void put32(std::vector<uint8_t>& v, size_t at, uint32_t x) { std::memcpy(&v[at], &x, 4); }
static inline void put16(std::vector<uint8_t>& v, size_t at, uint16_t x) { std::memcpy(&v[at], &x, 2); }

static int64_t ans_encode(const uint8_t* sym, int64_t n, uint8_t* out, int64_t cap) {
  const int64_t nc = (n + kAnsChunk - 1) / kAnsChunk;
  uint64_t count[2][256] = {};
  for (int64_t i = 0; i < n; ++i) ++count[i & 1][sym[i]];
  uint16_t freq[2][256];
  uint32_t start[2][256];
  for (int k = 0; k < 2; ++k) {
    ans_quantize(count[k], freq[k]);
    uint32_t acc = 0;
    for (int s = 0; s < 256; ++s) {
      start[k][s] = acc;
      acc += freq[k][s];
    }
  }
  std::vector<uint8_t> buf(static_cast<size_t>(ans_header_bytes(nc)), 0);
  put32(buf, 0, kAnsMagic);
  put32(buf, 4, static_cast<uint32_t>(n));
  put32(buf, 8, static_cast<uint32_t>(nc));
  for (int k = 0; k < 2; ++k)
    for (int s = 0; s < 256; ++s) put16(buf, 16 + 2 * (k * 256 + s), freq[k][s]);
  std::vector<uint16_t> words;
  for (int64_t c = 0; c < nc; ++c) {
    const size_t at = buf.size();
    put32(buf, kAnsHeader + 4 * c, static_cast<uint32_t>(at));
    const int64_t base = c * kAnsChunk;
    const int cnt = static_cast<int>(std::min<int64_t>(kAnsChunk, n - base));
    buf.resize(at + kAnsChunkHdr, 0);
    for (int w = 0; w < kAnsWays; ++w) {
      const int k = w & 1;
      words.clear();
      uint32_t x = kAnsLow;
      for (int j = ans_stream_symbols(cnt, w) - 1; j >= 0; --j) {  // encode in reverse order
        const uint8_t s = sym[base + w + static_cast<int64_t>(j) * kAnsWays];
        const uint32_t f = freq[k][s];
        if (x >= (f << 20)) {
          words.push_back(static_cast<uint16_t>(x & 0xffffu));
          x >>= 16;
        }
        x = ((x / f) << kAnsScale) + x % f + start[k][s];
      }
      put32(buf, at + 4 * w, x);
      put16(buf, at + 4 * kAnsWays + 2 * w, static_cast<uint16_t>(words.size()));
      const size_t w0 = buf.size();
      buf.resize(w0 + 2 * words.size());
      for (size_t q = 0; q < words.size(); ++q) put16(buf, w0 + 2 * q, words[words.size() - 1 - q]);
    }
    buf.resize((buf.size() + 15) / 16 * 16, 0);
  }
  put32(buf, kAnsHeader + 4 * nc, static_cast<uint32_t>(buf.size()));
  if (static_cast<int64_t>(buf.size()) > cap) return -1;
  std::memcpy(out, buf.data(), buf.size());
  return static_cast<int64_t>(buf.size());
}

// ---- GPU decoder ------------------------------------------------------------------------------
// One launch decodes a list of segments (<= 32) of one source buffer into one destination: kind 0
// segments are VQ2A streams, kind 1 segments are stored bytes (copied). An ANS-coded expert
// record is four segments (gate_up indices, gate_up scales, down indices, down scales), so a paged
// miss is one H2D copy of the compressed record and one launch that writes the whole slot.
//
// ANS segments: one warp per chunk, 4 warps per CTA, lane l running streams l and l + 32 side by
// side (two independent dependency chains; both streams have parity l & 1, hence one context).
// The CTA builds, for both contexts, a 4096-entry table in shared memory holding per slot
// (symbol | freq << 8 | (slot - start) << 20), so a step is one shared load and one multiply-add:
// x = freq * (x >> 12) + (slot - start). The warp first stages the chunk's words in shared memory
// with coalesced loads; the renormalisation step is branch-free (the next word is read every
// step, used when x < L). Every offset read from the stream is checked against the segment's
// length before use; a malformed stream raises *status (atomicMax of an error code), and its
// lanes stop or run on harmlessly, never reading or writing out of bounds.
enum AnsError { kAnsOk = 0, kAnsBadMagic = 1, kAnsBadCount = 2, kAnsBadFreq = 3, kAnsBadChunk = 4,
                kAnsBadWords = 5, kAnsUnderflow = 6, kAnsBadFinal = 7 };
enum AnsKind { kSegAns = 0, kSegStored = 1 };
constexpr int kAnsMaxSegs = 32;  // 8 expert records of 4 segments
constexpr int kAnsWarps = 4;
constexpr int kStoredBlockBytes = 128 * 16 * 4;  // bytes one CTA copies for a stored segment
constexpr int kWordStage = 2 * kAnsChunk + 16;   // a chunk's words (<= one per symbol) + slack
constexpr int kAnsSmem = 2 * kAnsTotal * 4 + kAnsWarps * kWordStage;  // slot tables + word stages

struct AnsSegs {
  const uint8_t* src[kAnsMaxSegs];
  uint8_t* dst[kAnsMaxSegs];
  int64_t bytes[kAnsMaxSegs];   // segment length in the source
  int64_t n[kAnsMaxSegs];       // decoded length (== bytes for stored segments)
  int32_t kind[kAnsMaxSegs];
  int32_t vec[kAnsMaxSegs];     // stored segment copyable with 16-byte vectors
  int32_t block0[kAnsMaxSegs + 1];
  int32_t nseg;
};

__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}
__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
}

__device__ void stored_copy(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t n, bool vec,
                            int64_t b) {
  const int64_t lo = b * kStoredBlockBytes, hi = min(n, lo + kStoredBlockBytes);
  if (vec) {
    for (int64_t i = lo + 16 * threadIdx.x; i < hi; i += 16 * blockDim.x)
      *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src + i);
  } else {
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = src[i];
  }
}

// One decode step of one stream; returns the symbol. w: the stream's staged words, i: words
// consumed so far (never beyond nw; w[nw] lies inside the stage), under: set when words run out.
__device__ __forceinline__ uint32_t ans_step(const uint32_t* __restrict__ tab, uint32_t& x,
                                             const uint16_t* __restrict__ w, uint32_t& i, uint32_t nw,
                                             uint32_t& under) {
  const uint32_t nxt = w[i];
  const uint32_t e = tab[x & (kAnsTotal - 1)];
  x = ((e >> 8) & 0xfffu) * (x >> kAnsScale) + (e >> 20);
  const bool renorm = x < kAnsLow;
  const bool have = i < nw;
  under |= static_cast<uint32_t>(renorm && !have);
  x = renorm ? (x << 16) | nxt : x;
  i += static_cast<uint32_t>(renorm && have);
  return e & 0xffu;
}

__global__ void __launch_bounds__(128) ans_decode_kernel(AnsSegs a, int32_t* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t dsmem[];
  uint32_t (*table)[kAnsTotal] = reinterpret_cast<uint32_t (*)[kAnsTotal]>(dsmem);  // 32 KB
  __shared__ uint32_t cum[2][257];
  __shared__ uint32_t starts[2][kAnsTotal / 32];  // bit q set: a symbol's slot range starts at q
  __shared__ uint32_t wsum[kAnsWarps];
  __shared__ int bad;
  pdl_wait();
  int sg = 0;
  while (sg + 1 < a.nseg && static_cast<int>(blockIdx.x) >= a.block0[sg + 1]) ++sg;
  const int64_t b = static_cast<int64_t>(blockIdx.x) - a.block0[sg];
  const uint8_t* in = a.src[sg];
  if (a.kind[sg] == kSegStored) {
    stored_copy(in, a.dst[sg], a.n[sg], a.vec[sg] != 0, b);
    return;
  }
  const int64_t nbytes = a.bytes[sg], n = a.n[sg];
  const int64_t nc = (n + kAnsChunk - 1) / kAnsChunk;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Frequencies -> cumulative starts, all threads at once: context k = tid / 64, thread t of the
  // context holds symbols 4t .. 4t+3 (the host checked the header lies inside the segment).
  const int k = tid >> 6, t = tid & 63;
  uint32_t f[4], run = 0;
  bool zero = false;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[j] = ld_u16(in + 16 + 2 * (k * 256 + 4 * t + j));
    zero |= f[j] == 0;
    run += f[j];
  }
  uint32_t incl = run;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  starts[k][2 * t] = 0;
  starts[k][2 * t + 1] = 0;
  if (tid == 0) {
    int h = kAnsOk;
    if (ld_u32(in) != kAnsMagic) h = kAnsBadMagic;
    else if (ld_u32(in + 4) != static_cast<uint32_t>(n) || ld_u32(in + 8) != static_cast<uint32_t>(nc))
      h = kAnsBadCount;
    bad = h;
  }
  __syncthreads();
  const uint32_t total = wsum[2 * k] + wsum[2 * k + 1];
  if (zero || total != kAnsTotal) atomicMax(&bad, kAnsBadFreq);
  uint32_t c0 = incl - run + ((warp & 1) ? wsum[warp - 1] : 0u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    cum[k][4 * t + j] = c0;
    if (c0 < kAnsTotal) atomicOr(&starts[k][c0 >> 5], 1u << (c0 & 31));  // table built only if valid
    c0 += f[j];
  }
  if (t == 63) cum[k][256] = total;
  __syncthreads();
  if (bad != kAnsOk) {
    if (tid == 0) atomicMax(status, bad);
    return;
  }
  {  // slot table: thread t of context k fills slots 64t .. 64t+63
    const uint32_t s0 = 64u * t;
    int lo = 0, hi = 255;  // the symbol owning slot s0: last s with cum[s] <= s0
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cum[k][mid] <= s0) lo = mid;
      else hi = mid - 1;
    }
    uint32_t s = lo, st = cum[k][lo];
    const uint64_t bits = static_cast<uint64_t>(starts[k][2 * t]) | (static_cast<uint64_t>(starts[k][2 * t + 1]) << 32);
#pragma unroll 16
    for (int q = 0; q < 64; ++q) {
      if (q > 0 && ((bits >> q) & 1u)) {
        ++s;
        st = s0 + q;
      }
      const uint32_t fs = cum[k][s + 1] - st;
      table[k][s0 + q] = s | (fs << 8) | ((s0 + q - st) << 20);
    }
  }
  __syncthreads();

  const int64_t c = b * kAnsWarps + warp;
  if (c >= nc) return;
  const int64_t o0 = ld_u32(in + kAnsHeader + 4 * c);
  const int64_t o1 = ld_u32(in + kAnsHeader + 4 * (c + 1));
  int err = kAnsOk;
  if (o0 < ans_header_bytes(nc) || o0 + kAnsChunkHdr > o1 || o1 > nbytes) err = kAnsBadChunk;
  err = __reduce_max_sync(0xffffffffu, err);
  if (err != kAnsOk) {
    if (lane == 0) atomicMax(status, err);
    return;
  }
  const int cnt = static_cast<int>(min(static_cast<int64_t>(kAnsChunk), n - c * kAnsChunk));
  const int ma = ans_stream_symbols(cnt, lane), mb = ans_stream_symbols(cnt, lane + 32);
  uint32_t xa = ld_u32(in + o0 + 4 * lane), xb = ld_u32(in + o0 + 4 * (lane + 32));
  const uint32_t na = ld_u16(in + o0 + 4 * kAnsWays + 2 * lane);
  const uint32_t nb = ld_u16(in + o0 + 4 * kAnsWays + 2 * (lane + 32));
  if (na > static_cast<uint32_t>(ma) || nb > static_cast<uint32_t>(mb)) err = kAnsBadWords;
  err = __reduce_max_sync(0xffffffffu, err);
  if (err != kAnsOk) {
    if (lane == 0) atomicMax(status, err);
    return;
  }
  // word offsets: streams 0..31 (the lanes' first streams) come first, then streams 32..63
  uint32_t pa = na, pb = nb;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t va = __shfl_up_sync(0xffffffffu, pa, d), vb = __shfl_up_sync(0xffffffffu, pb, d);
    if (lane >= d) {
      pa += va;
      pb += vb;
    }
  }
  const uint32_t tot_a = __shfl_sync(0xffffffffu, pa, 31);
  const uint32_t words = tot_a + __shfl_sync(0xffffffffu, pb, 31);  // <= 8192: counts <= symbols
  pa -= na;
  pb += tot_a - nb;
  if (static_cast<uint64_t>(o0) + kAnsChunkHdr + 2ull * words > static_cast<uint64_t>(o1)) {
    if (lane == 0) atomicMax(status, kAnsBadWords);
    return;
  }
  // Stage the chunk's words (<= 16 KB) in this warp's shared buffer with coalesced loads.
  uint8_t* stage = dsmem + 2 * kAnsTotal * 4 + warp * kWordStage;
  const uint8_t* gw = in + o0 + kAnsChunkHdr;
  const int wbytes = 2 * static_cast<int>(words);
  int done = 0;
  if (aligned(gw, 16)) {
    done = wbytes & ~15;
    for (int i = 16 * lane; i < done; i += 16 * 32)
      *reinterpret_cast<uint4*>(stage + i) = __ldg(reinterpret_cast<const uint4*>(gw + i));
  }
  for (int i = done + lane; i < wbytes; i += 32) stage[i] = gw[i];
  __syncwarp();
  const uint16_t* wa = reinterpret_cast<const uint16_t*>(stage) + pa;
  const uint16_t* wb = reinterpret_cast<const uint16_t*>(stage) + pb;
  const uint32_t* tab = table[lane & 1];
  uint8_t* out = a.dst[sg] + c * kAnsChunk + lane;
  uint32_t ia = 0, ib = 0, under = 0;
  int j = 0;
#pragma unroll 4
  for (; j < mb; ++j) {
    const uint32_t sa = ans_step(tab, xa, wa, ia, na, under);
    const uint32_t sb = ans_step(tab, xb, wb, ib, nb, under);
    out[j * kAnsWays] = static_cast<uint8_t>(sa);
    out[j * kAnsWays + 32] = static_cast<uint8_t>(sb);
  }
  if (j < ma) {  // stream a holds one more symbol than stream b in a partial last chunk
    const uint32_t sa = ans_step(tab, xa, wa, ia, na, under);
    out[j * kAnsWays] = static_cast<uint8_t>(sa);
  }
  if (under) err = kAnsUnderflow;
  else if (xa != kAnsLow || xb != kAnsLow || ia != na || ib != nb) err = kAnsBadFinal;
  if (err != kAnsOk) atomicMax(status, err);
}

// Validate the segment list, fill the kernel parameters and launch (also used by the pager).
int ans_launch(const uint8_t* src, int64_t src_bytes, const int64_t* src_off, const int64_t* seg_bytes,
                      const int64_t* dst_off, const int64_t* seg_n, const int32_t* kind, int64_t nseg, uint8_t* dst,
                      int64_t dst_bytes, int32_t* status, cudaStream_t st) {
  if (!src || !dst || !status || !src_off || !seg_bytes || !dst_off || !seg_n || !kind) return VQ2_ERR_ARG;
  if (nseg < 1 || nseg > kAnsMaxSegs || src_bytes < 0 || dst_bytes < 0) return VQ2_ERR_ARG;
  AnsSegs a = {};
  int64_t blocks = 0;
  for (int i = 0; i < nseg; ++i) {
    const int64_t so = src_off[i], sb = seg_bytes[i], d0 = dst_off[i], n = seg_n[i];
    if (so < 0 || sb < 0 || d0 < 0 || n < 0 || so > src_bytes - sb || d0 > dst_bytes - n) return VQ2_ERR_SHAPE;
    a.src[i] = src + so;
    a.dst[i] = dst + d0;
    a.bytes[i] = sb;
    a.n[i] = n;
    a.kind[i] = kind[i];
    a.block0[i] = static_cast<int32_t>(blocks);
    if (kind[i] == kSegAns) {
      if (n > INT32_MAX) return VQ2_ERR_SHAPE;
      const int64_t nc = (n + kAnsChunk - 1) / kAnsChunk;
      if (nc > 0 && sb < ans_header_bytes(nc)) return VQ2_ERR_SHAPE;
      blocks += (nc + kAnsWarps - 1) / kAnsWarps;
    } else if (kind[i] == kSegStored) {
      if (sb != n) return VQ2_ERR_SHAPE;
      a.vec[i] = aligned(a.src[i], 16) && aligned(a.dst[i], 16) && n % 16 == 0;
      blocks += (n + kStoredBlockBytes - 1) / kStoredBlockBytes;
    } else {
      return VQ2_ERR_ARG;
    }
    if (blocks > INT32_MAX) return VQ2_ERR_SHAPE;
  }
  a.block0[nseg] = static_cast<int32_t>(blocks);
  a.nseg = static_cast<int32_t>(nseg);
  if (blocks == 0) return VQ2_OK;
  static std::atomic<uint64_t> attr_done{0};  // per-device dynamic shared memory opt-in
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(attr_done.load() & bit)) {
    const cudaError_t e = cudaFuncSetAttribute(ans_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAnsSmem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return VQ2_ERR_LAUNCH;
    }
    attr_done.fetch_or(bit);
  }
  return launch_kernel(ans_decode_kernel, dim3(static_cast<unsigned>(blocks)), dim3(128), kAnsSmem, st, a, status);
}

}  // namespace vq2

extern "C" int64_t vq2_rans_bound(int64_t n_symbols) {
  if (n_symbols < 0 || n_symbols > INT32_MAX) return -1;
  return vq2::ans_bound(n_symbols);
}

extern "C" int vq2_rans_encode(const uint8_t* symbols, int64_t n_symbols, uint8_t* out, int64_t out_capacity,
                               int64_t* out_bytes) {
  if ((!symbols && n_symbols > 0) || !out || !out_bytes) return VQ2_ERR_ARG;
  if (n_symbols < 0 || n_symbols > INT32_MAX) return VQ2_ERR_SHAPE;
  const int64_t got = vq2::ans_encode(symbols, n_symbols, out, out_capacity);
  if (got < 0) return VQ2_ERR_ARG;  // capacity below the encoded size
  *out_bytes = got;
  return VQ2_OK;
}

extern "C" int vq2_rans_decode(const void* stream, int64_t stream_bytes, int64_t n_symbols, void* out,
                               int64_t out_capacity, int32_t* status, void* cuda_stream) {
  const int64_t off = 0;
  const int32_t kind = vq2::kSegAns;
  return vq2::ans_launch(static_cast<const uint8_t*>(stream), stream_bytes, &off, &stream_bytes, &off, &n_symbols,
                         &kind, 1, static_cast<uint8_t*>(out), out_capacity, status,
                         static_cast<cudaStream_t>(cuda_stream));
}

extern "C" int vq2_rans_decode_segments(const void* src, int64_t src_bytes, const int64_t* seg_src_off,
                                        const int64_t* seg_src_bytes, const int64_t* seg_dst_off,
                                        const int64_t* seg_n, const int32_t* seg_kind, int64_t nseg, void* dst,
                                        int64_t dst_bytes, int32_t* status, void* cuda_stream) {
  return vq2::ans_launch(static_cast<const uint8_t*>(src), src_bytes, seg_src_off, seg_src_bytes, seg_dst_off, seg_n,
                         seg_kind, nseg, static_cast<uint8_t*>(dst), dst_bytes, status,
                         static_cast<cudaStream_t>(cuda_stream));
}
