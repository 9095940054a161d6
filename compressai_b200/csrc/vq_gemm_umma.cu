// Batched VQ GEMV on the 5th-generation tensor cores of sm_100a: tcgen05.mma with its fp32
// accumulator in tensor memory (TMEM), the activation operand brought into shared memory by TMA
// (cp.async.bulk.tensor, 128-byte swizzle), and the weight operand decoded from the codebook by
// the CTA's own warps straight into the same swizzled layout.
//
//   y[m, r] = rs * scale[r] * sum_k W[r, k] * x[m, k],  W[r, 8g + t] = cb0[idx0[r, g]][t] (+ cb1[idx1[r, g]][t])
//
// Work item: 128 weight rows (the MMA's M) x one tile of NT tokens (the MMA's N, 16..128), K
// walked in chunks of 64 (one 128-byte swizzle row of 16-bit values, 8 index groups). Roles:
//   * warps 0-7, two groups of four (even / odd chunks): each thread owns one weight row of its
//     group's chunks -- one 16-byte index load (prefetched one chunk ahead), 8 random 16-byte
//     codebook gathers (L2 evict-last, issued before the wait for the stage), then the row's 64
//     decoded values into the stage's A operand: by default one tcgen05.st into tensor memory
//     (row -> TMEM lane, two 16-bit K values per 32-bit column), else 8 bank-conflict-free
//     16-byte stores into a 128-byte-swizzled shared-memory tile and a proxy fence; then one
//     mbarrier arrival per warp. The group's first thread also starts the TMA copy of the
//     chunk's activation tile (NT x 64) into the stage's B tile in shared memory;
//   * warp 8 allocates the TMEM columns (two accumulators of NT columns: the epilogue of one
//     item runs while the next item accumulates; plus the A stages when A lives in TMEM) and its
//     lane 0 issues the MMAs, 4 x (K = 16) per chunk,
//     once the stage's gathers and its TMA copy have landed, then commits the stage back to its
//     producers (tcgen05.commit -> mbarrier);
//   * warps 9-12: epilogue -- tcgen05.ld of their 32-lane quarter of the accumulator (one weight
//     row per thread, 16 token columns per load), row scale, stores of 32 consecutive rows per
//     warp instruction.
// The op stays bound by the codebook gathers (one L1TEX line per codeword at any M), so the MMA
// issue rate only has to keep pace; the tensor pipe does in one instruction what the CUDA-core
// kernel does with 8*M FMAs per codeword.
//
// Precision: fp16 codebooks take the activations rounded once to fp16 (one MMA per K step;
// max|y - y_fp64| / max|y| is ~2e-4, inside the 1e-3 bar); bf16 codebooks split the activations
// into bf16 hi + lo halves and run two MMAs per K step (bf16 alone would cost ~1e-3).
//
// Waits: every mbarrier wait is bounded (kUmWaitCycles). A wait that gives up raises the
// CTA's abort flag and VQ2_ERR_TIMEOUT in the device status word g_umma_status (read by
// vq2_tc_status); every role then leaves its loop, the MMA thread waits (bounded) for its
// issued MMAs, each TMA issuer for its copies in flight, and TMEM is freed before the CTA exits.
//
// Semantics: the batched form of reference vq2/kernels.py:32-78 (whose Triton path serves
// M = 1 only; vq2/runtime.py:105-110 dequantizes and calls F.linear for M > 1).
#include <cuda.h>  // CUtensorMap and its enums (the encoder is fetched from the driver at run time)

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "gemv_dev.cuh"

// Sticky status of the tcgen05 GEMV: VQ2_ERR_TIMEOUT once any bounded wait gave up.
__device__ int32_t g_umma_status;

namespace vq2 {
namespace {

constexpr int kUmKC = 64;                  // K elements per chunk (one 128-byte row of 16-bit values)
constexpr int kUmRows = 128;               // weight rows per tile = MMA M
constexpr int kUmMmaWarp = 8;              // TMEM owner, MMA issuer (lane 0)
constexpr int kUmEpiWarp0 = 9;             // warps 9..12: epilogue
constexpr int kUmThreads = 13 * 32;
static_assert(kUmEpiWarp0 == kUmMmaWarp + 1 && kUmThreads == (kUmEpiWarp0 + 4) * 32, "warp roles");
constexpr long long kUmWaitCycles = 4000000000LL;  // ~2 s at 1.965 GHz

// ---- PTX wrappers ------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Generic-proxy writes to shared memory become visible to the async proxy (tensor core, TMA).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte swizzle layout: rows
// of 128 bytes, 8-row groups 1024 bytes apart (SBO), tile base 1024-byte aligned. Bits: start
// address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused by this layout: 1), stride byte
// offset >> 4 [32,46), descriptor version 1 [46,48), layout 2 = 128-byte swizzle [61,64).
// Advancing K by 16 elements (32 bytes) inside the swizzle row adds 2 to the address field.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor of kind::f16: D fp32 [4,6) = 1, A / B type [7,10) / [10,13) (0 fp16,
// 1 bf16), both K-major (bits 15, 16 = 0), N >> 3 at [17,23), M >> 4 at [24,29).
template <int N, bool BF16>
constexpr uint32_t umma_idesc() {
  return (1u << 4) | ((BF16 ? 1u : 0u) << 7) | ((BF16 ? 1u : 0u) << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(kUmRows >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  const uint32_t z = 0;  // no output lanes disabled
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}
// The same MMA with the A operand read from tensor memory (lane = row, 16-bit K values packed two
// per 32-bit column, K = 16 per instruction = 8 columns).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}

// This thread's 32 consecutive 32-bit TMEM columns of its lane (32x32b shape; warp-collective),
// waited for before returning.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint4 (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
      "tcgen05.wait::st.sync.aligned;"
      ::"r"(taddr), "r"(v[0].x), "r"(v[0].y), "r"(v[0].z), "r"(v[0].w), "r"(v[1].x), "r"(v[1].y), "r"(v[1].z),
        "r"(v[1].w), "r"(v[2].x), "r"(v[2].y), "r"(v[2].z), "r"(v[2].w), "r"(v[3].x), "r"(v[3].y), "r"(v[3].z),
        "r"(v[3].w), "r"(v[4].x), "r"(v[4].y), "r"(v[4].z), "r"(v[4].w), "r"(v[5].x), "r"(v[5].y), "r"(v[5].z),
        "r"(v[5].w), "r"(v[6].x), "r"(v[6].y), "r"(v[6].z), "r"(v[6].w), "r"(v[7].x), "r"(v[7].y), "r"(v[7].z),
        "r"(v[7].w)
      : "memory");
}

// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (32x32b shape), waited for in the same
// statement so no use of the registers can move ahead of the wait.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared control block: per stage, the producers' arrivals (4 warps), the TMA copy (one arrival
// + transaction bytes) and the MMA's release; per accumulator, "MMAs done" and "epilogue done".
template <int S>
struct UmCtl {
  uint64_t full[S], tma[S], empty[S], done[2], drained[2], drain;
  uint32_t tmem_base;
  int abort;
};

template <int S>
__device__ __forceinline__ void um_fail(UmCtl<S>* ctl) {
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
  atomicMax(&g_umma_status, VQ2_ERR_TIMEOUT);
}

// Bounded wait on (bar, parity); false when this CTA aborted (here or elsewhere).
template <int S>
__device__ __forceinline__ bool um_wait(uint32_t bar, uint32_t parity, UmCtl<S>* ctl) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (*reinterpret_cast<volatile int*>(&ctl->abort)) return false;
    if (clock64() - t0 > kUmWaitCycles) {
      um_fail(ctl);
      return false;
    }
  }
  return true;
}
// Bounded wait used while draining after an abort (ignores the abort flag).
__device__ __forceinline__ bool um_drain(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity))
    if (clock64() - t0 > kUmWaitCycles) return false;
  return true;
}

// The CTA's contiguous range of items (one CTA per SM): a floor / ceil split.
__device__ __forceinline__ void um_items(int64_t items, int64_t& lo, int64_t& hi) {
  const int64_t G = gridDim.x, b = blockIdx.x;
  lo = b * items / G;
  hi = (b + 1) * items / G;
}

struct UmItem {
  int p, rb, m0, out;
};
__device__ __forceinline__ UmItem um_decode(const GemvArgs& a, int64_t it, int NT) {
  UmItem w;
  const int mt = (int)(it / a.row_blocks);
  const int rbg = (int)(it - (int64_t)mt * a.row_blocks);
  int p = 0;
#pragma unroll 1
  while (p + 1 < a.nprob && rbg >= a.p_rb0[p + 1]) ++p;
  w.p = p;
  w.rb = rbg - a.p_rb0[p];
  w.m0 = mt * NT;
  w.out = a.p_out[p];
  return w;
}

// Columns of a TMEM allocation: a power of two from 32 to 512.
constexpr uint32_t tmem_cols(uint32_t need) {
  return need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128 : need <= 256 ? 256 : 512;
}

// AT: the decoded weight tile (MMA operand A) is written to tensor memory by the producers
// (tcgen05.st) instead of to shared memory. Stage s's A tile then occupies TMEM columns
// [2 NT + 32 s, +32) of all 128 lanes, and shared memory only carries the activation tiles.
template <int NT, int S, bool RES, bool LO, typename TV, bool AT>
__global__ void __launch_bounds__(kUmThreads, 1) vq_umma_kernel(const GemvArgs a, const __grid_constant__ CUtensorMap xmap,
                                                                 const __grid_constant__ CUtensorMap lmap) {
  constexpr int A_BYTES = AT ? 0 : kUmRows * 128;
  constexpr int B_BYTES = NT * 128;
  constexpr int STAGE = A_BYTES + B_BYTES * (LO ? 2 : 1);
  constexpr uint32_t ACC_COLS = 2 * NT;                 // two accumulators of NT fp32 columns
  constexpr uint32_t A_COL0 = ACC_COLS;                 // AT: first column of the A stages
  constexpr uint32_t NEED_COLS = ACC_COLS + (AT ? 32u * S : 0u);
  constexpr uint32_t TMEM_COLS = tmem_cols(NEED_COLS);
  constexpr uint32_t IDESC = umma_idesc<NT, std::is_same<TV, __nv_bfloat16>::value>();
  static_assert(NEED_COLS <= 512, "accumulators and A stages exceed tensor memory");
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "swizzled tiles must stay 1024-byte aligned");
  static_assert(S % 2 == 0, "each producer group owns every other stage");
  extern __shared__ unsigned char um_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(um_raw) + 1023) & ~uintptr_t(1023));
  uint4* cb1s = reinterpret_cast<uint4*>(sm + S * STAGE);
  UmCtl<S>* ctl = reinterpret_cast<UmCtl<S>*>(sm + S * STAGE + (RES ? 4096 : 0));
  auto stage_a = [&](int s) { return sm + s * STAGE; };
  auto stage_b = [&](int s) { return sm + s * STAGE + A_BYTES; };
  auto stage_bl = [&](int s) { return sm + s * STAGE + A_BYTES + B_BYTES; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = a.n / kUmKC;
  const int64_t items = (int64_t)a.row_blocks * a.mtiles;
  int64_t i0, i1;
  um_items(items, i0, i1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(su32(&ctl->full[s]), 4);
      mbar_init(su32(&ctl->tma[s]), 1);
      mbar_init(su32(&ctl->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(su32(&ctl->done[b]), 1);
      mbar_init(su32(&ctl->drained[b]), 4);
    }
    mbar_init(su32(&ctl->drain), 1);
    ctl->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_proxy_async();
  }
  if (RES)
    for (int i = threadIdx.x; i < 256; i += blockDim.x) cb1s[i] = static_cast<const uint4*>(a.cb1)[i];
  if (warp == kUmMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&ctl->tmem_base)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp < 8) {
    // ---------------------------------------------------------------------------- producers
    const int grp = warp >> 2;            // this group fills the even (0) or odd (1) chunks
    const int r = threadIdx.x & 127;      // weight row of the tile
    const bool leader = r == 0;           // issues the group's TMA copies
    const uint64_t pol_s = policy_evict_first();
    const uint64_t pol_c = policy_evict_last();
    const uint4* cb0 = static_cast<const uint4*>(a.cb0);
    const int ng = a.n >> 3;
    uint32_t issued_use[S];               // last use of each stage whose TMA this leader started (+1)
#pragma unroll
    for (int s = 0; s < S; ++s) issued_use[s] = 0;

    // index vector of (item it, chunk c) for this thread's row; zero past the matrix
    auto load_iv = [&](int64_t it, int c, uint4& iv, uint2& jv) {
      iv = make_uint4(0, 0, 0, 0);
      jv = make_uint2(0, 0);
      if (it >= i1) return;
      const UmItem w = um_decode(a, it, NT);
      const int row = w.rb * kUmRows + r;
      if (row >= w.out) return;
      const int64_t off = (int64_t)row * ng + c * 8;
      iv = ld_stream_u4(a.p_idx0[w.p] + off, pol_s);
      if (RES) jv = ld_stream_u2(a.p_idx1[w.p] + off, pol_s);
    };
    uint4 iv;
    uint2 jv;
    load_iv(i0, grp, iv, jv);  // constant weights: before the dependency wait
    pdl_wait();
    pdl_trigger();
    int il = 0;
    for (int64_t it = i0; it < i1; ++it, ++il) {
      const UmItem w = um_decode(a, it, NT);
      const bool row_ok = w.rb * kUmRows + r < w.out;
      for (int c = grp; c < chunks; c += 2) {
        // prefetch the next chunk of this group (possibly the next item's first)
        uint4 niv;
        uint2 njv;
        if (c + 2 < chunks) load_iv(it, c + 2, niv, njv);
        else load_iv(it + 1, grp, niv, njv);
        const uint32_t gc = (uint32_t)il * chunks + c;
        const int s = (int)(gc % S);
        const uint32_t u = gc / S;
        // the gathers go out first: their L2 round trip overlaps the wait for the stage
        uint4 cw[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t w32 = (&iv.x)[j >> 1];
          const uint32_t code = (j & 1) ? (w32 >> 16) : (w32 & 0xffffu);
          cw[j] = row_ok ? ld_cb_u4(cb0 + code, pol_c) : make_uint4(0, 0, 0, 0);
        }
        {
          const bool ok = um_wait(su32(&ctl->empty[s]), (u & 1) ^ 1, ctl);
          if (!__all_sync(0xffffffffu, ok)) goto producer_exit;  // warp-uniform (tcgen05.st is collective)
        }
        if (leader) {
          mbar_arrive_tx(su32(&ctl->tma[s]), B_BYTES * (LO ? 2 : 1));
          tma_load_2d(su32(stage_b(s)), &xmap, c * kUmKC, w.m0, su32(&ctl->tma[s]));
          if (LO) tma_load_2d(su32(stage_bl(s)), &lmap, c * kUmKC, w.m0, su32(&ctl->tma[s]));
          issued_use[s] = u + 1;
        }
        if (RES) {  // 3 bpw: cb0 + cb1 summed in fp32 and rounded once to the operand type
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t b = ((&jv.x)[j >> 2] >> ((j & 3) * 8)) & 0xffu;
            float f0[8], f1[8];
            decode8<TV>(cw[j], f0);
            decode8<TV>(cb1s[b], f1);
            TV o[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) o[t] = from_f32<TV>(f0[t] + f1[t]);
            cw[j] = row_ok ? *reinterpret_cast<const uint4*>(o) : make_uint4(0, 0, 0, 0);
          }
        }
        if constexpr (AT) {
          // row r -> TMEM lane r (this warp's lane quarter), K values 2c, 2c+1 -> column c
          tc_fence_after();
          tmem_st32(tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + A_COL0 + 32u * s, cw);
          tc_fence_before();
        } else {
          unsigned char* A = stage_a(s) + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(A + ((j ^ (r & 7)) << 4)) = cw[j];
          fence_proxy_async();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(su32(&ctl->full[s]));
        iv = niv;
        jv = njv;
      }
    }
  producer_exit:
    if (leader) {  // copies this thread started have landed before the CTA's shared memory goes away
#pragma unroll
      for (int s = 0; s < S; ++s)
        if (issued_use[s] && !um_drain(su32(&ctl->tma[s]), (issued_use[s] - 1) & 1))
          atomicMax(&g_umma_status, VQ2_ERR_TIMEOUT);
    }
  } else if (warp == kUmMmaWarp) {
    // ---------------------------------------------------------------------------- MMA issuer
    pdl_wait();
    pdl_trigger();
    if (lane == 0) {
      int il = 0;
      bool ok = true;
      for (int64_t it = i0; it < i1 && ok; ++it, ++il) {
        const int b = il & 1;
        const uint32_t ub = (uint32_t)il >> 1;
        if (il >= 2 && !um_wait(su32(&ctl->drained[b]), (ub - 1) & 1, ctl)) break;  // epilogue of item il-2 read it
        tc_fence_after();
        const uint32_t d = tmem + b * NT;
        for (int c = 0; c < chunks; ++c) {
          const uint32_t gc = (uint32_t)il * chunks + c;
          const int s = (int)(gc % S);
          const uint32_t u = gc / S;
          if (!um_wait(su32(&ctl->full[s]), u & 1, ctl) || !um_wait(su32(&ctl->tma[s]), u & 1, ctl)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bd = sw128_desc(su32(stage_b(s)));
          if constexpr (AT) {
            const uint32_t at = tmem + A_COL0 + 32u * s;
#pragma unroll
            for (int kk = 0; kk < kUmKC / 16; ++kk) umma_f16_ts(d, at + 8 * kk, bd + 2 * kk, IDESC, (c | kk) != 0);
            if (LO) {
              const uint64_t bl = sw128_desc(su32(stage_bl(s)));
#pragma unroll
              for (int kk = 0; kk < kUmKC / 16; ++kk) umma_f16_ts(d, at + 8 * kk, bl + 2 * kk, IDESC, 1);
            }
          } else {
            const uint64_t ad = sw128_desc(su32(stage_a(s)));
#pragma unroll
            for (int kk = 0; kk < kUmKC / 16; ++kk) umma_f16(d, ad + 2 * kk, bd + 2 * kk, IDESC, (c | kk) != 0);
            if (LO) {
              const uint64_t bl = sw128_desc(su32(stage_bl(s)));
#pragma unroll
              for (int kk = 0; kk < kUmKC / 16; ++kk) umma_f16(d, ad + 2 * kk, bl + 2 * kk, IDESC, 1);
            }
          }
          umma_commit(su32(&ctl->empty[s]));
        }
        if (ok) umma_commit(su32(&ctl->done[b]));
      }
      // every MMA issued so far has completed before TMEM is freed
      umma_commit(su32(&ctl->drain));
      if (!um_drain(su32(&ctl->drain), 0)) atomicMax(&g_umma_status, VQ2_ERR_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------------------- epilogue
    pdl_wait();
    pdl_trigger();
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int il = 0;
    for (int64_t it = i0; it < i1; ++it, ++il) {
      const UmItem w = um_decode(a, it, NT);
      const int b = il & 1;
      const uint32_t ub = (uint32_t)il >> 1;
      if (!um_wait(su32(&ctl->done[b]), ub & 1, ctl)) break;
      tc_fence_after();
      const int row = w.rb * kUmRows + 32 * q + lane;
      const bool row_ok = row < w.out;
      const float sc = row_ok ? to_f32<TV>(static_cast<const TV*>(a.p_scale[w.p])[row]) * a.rs : 0.f;
      const int mcount = min(NT, a.M - w.m0);
      void* y = a.p_y[w.p];
#pragma unroll 1
      for (int j0 = 0; j0 < NT; j0 += 16) {
        float v[16];
        __syncwarp();  // tcgen05.ld is warp-collective
        tmem_ld16(tmem + (static_cast<uint32_t>(32 * q) << 16) + b * NT + j0, v);
        if (row_ok) {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int m = j0 + jj;
            if (m < mcount) {
              const int64_t o = (int64_t)(w.m0 + m) * a.y_row_stride + row;
              const float val = v[jj] * sc;
              if (a.y_dtype == VQ2_F16) static_cast<__half*>(y)[o] = __float2half_rn(val);
              else if (a.y_dtype == VQ2_BF16) static_cast<__nv_bfloat16*>(y)[o] = __float2bfloat16_rn(val);
              else static_cast<float*>(y)[o] = val;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(su32(&ctl->drained[b]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kUmMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---- host side ---------------------------------------------------------------------------------
// cuTensorMapEncodeTiled, fetched once from the driver (the library links only the CUDA runtime).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [rows, n] 16-bit row-major operand at `base`, boxes of NT rows x 64 elements, 128-byte swizzle
// (the UMMA K-major layout); rows past `rows` read as zeros.
bool make_operand_map(CUtensorMap* map, const void* base, int64_t rows, int64_t n, int NT, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(n * 2)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kUmKC), static_cast<cuuint32_t>(NT)};
  const cuuint32_t es[2] = {1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
            const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, int S, bool RES, bool LO, bool AT>
constexpr size_t umma_smem() {
  return 1024 + (size_t)S * ((AT ? 0 : kUmRows * 128) + NT * 128 * (LO ? 2 : 1)) + (RES ? 4096 : 0) +
         sizeof(UmCtl<S>);
}

// Where the decoded weight tile goes: tensor memory (default) or shared memory (VQ2_UMMA_A=smem).
bool umma_a_in_tmem() {
  static const bool on = [] {
    const char* v = std::getenv("VQ2_UMMA_A");
    return !(v && std::strcmp(v, "smem") == 0);
  }();
  return on;
}

template <int NT, bool RES, typename TV, bool AT>
int launch_umma(GemvArgs a, const void* xh, const void* xl, cudaStream_t st) {
  constexpr bool LO = std::is_same<TV, __nv_bfloat16>::value;
  // four stages (two per producer group) of at most 24 KB of shared memory each
  constexpr int S = AT || NT * 128 * (LO ? 2 : 1) <= 8192 ? 4 : 2;
  constexpr size_t smem = umma_smem<NT, S, RES, LO, AT>();
  auto kern = vq_umma_kernel<NT, S, RES, LO, TV, AT>;
  static std::atomic<uint64_t> done{0};
  static std::atomic<int> blocks_per_sm{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(done.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return VQ2_ERR_LAUNCH;
    }
    // One CTA per SM, and a shared-memory carveout just covering it. The gathers are served
    // through L1, and every codeword in flight holds an L1 line until it returns: with the SM's
    // whole shared memory configured (what the driver picked for this kernel when it ran two
    // CTAs per SM) only ~28 KB of L1 remained, which capped the gathers in flight per SM below
    // what the L2 round trip needs -- two CTAs per SM measured no faster than one.
    cudaFuncAttributes fa{};
    int smem_sm = 0, reserved = 0;
    e = cudaFuncGetAttributes(&fa, kern);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return VQ2_ERR_LAUNCH;
    }
    const int regs_warp = ((fa.numRegs * 32 + 255) / 256) * 256;       // allocation granularity
    const int by_regs = 65536 / (regs_warp * (kUmThreads / 32));
    const int by_smem = smem_sm / ((int)smem + reserved);
    if (by_regs < 1 || by_smem < 1) return VQ2_ERR_LAUNCH;
    const int nb = 1;
    // a hint: the driver rounds up to a supported configuration that holds the launch
    const int pct = (int)((((int64_t)smem + reserved) * nb * 100) / smem_sm);
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, pct > 100 ? 100 : pct);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return VQ2_ERR_LAUNCH;
    }
    blocks_per_sm.store(nb);
    done.fetch_or(bit);
  }
  CUtensorMap xmap, lmap;
  if (!make_operand_map(&xmap, xh, a.M, a.n, NT, LO)) return VQ2_ERR_LAUNCH;
  if (!make_operand_map(&lmap, LO ? xl : xh, a.M, a.n, NT, LO)) return VQ2_ERR_LAUNCH;
  const int64_t items = (int64_t)a.row_blocks * a.mtiles;
  const int64_t cap = (int64_t)sm_count() * blocks_per_sm.load();
  const int64_t grid = items < cap ? items : cap;
  if (grid <= 0) return VQ2_OK;
  return launch_kernel(kern, dim3((unsigned)grid), dim3(kUmThreads), smem, st, a, xmap, lmap);
}

template <bool RES, typename TV, bool AT>
int launch_umma_tile(const GemvArgs& a, const void* xh, const void* xl, cudaStream_t st) {
  if (a.M <= 16) return launch_umma<16, RES, TV, AT>(a, xh, xl, st);
  if (a.M <= 32) return launch_umma<32, RES, TV, AT>(a, xh, xl, st);
  if (a.M <= 64) return launch_umma<64, RES, TV, AT>(a, xh, xl, st);
  return launch_umma<128, RES, TV, AT>(a, xh, xl, st);
}

template <bool RES, typename TV>
int launch_umma_nt(const GemvArgs& a, const void* xh, const void* xl, cudaStream_t st) {
  return umma_a_in_tmem() ? launch_umma_tile<RES, TV, true>(a, xh, xl, st)
                          : launch_umma_tile<RES, TV, false>(a, xh, xl, st);
}

int token_tile(int64_t M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

bool umma_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("VQ2_UMMA");  // A/B switch: 0 keeps the mma.sync tensor-core kernel
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

}  // namespace

// Eligible: multi-matrix problems, n % 128 == 0, enough 128-row tiles to give every SM work
// (smaller matrices use the split-K mma.sync kernel), a workspace for the 16-bit operand(s).
int run_gemm_umma(const GemvArgs& a0, bool res, int val_dtype, void* ws, int64_t ws_bytes, cudaStream_t st) {
  if (!umma_enabled() || a0.nprob <= 0 || a0.n % 128 != 0 || ws == nullptr || a0.argmax) return -1;
  if (val_dtype != VQ2_F16 && val_dtype != VQ2_BF16) return -1;
  const bool lo = val_dtype == VQ2_BF16;
  const int64_t opnd = (int64_t)a0.M * a0.n * 2;
  if (ws_bytes < (lo ? 2 : 1) * opnd || !aligned(ws, 128)) return -1;
  GemvArgs a = a0;
  const int NT = token_tile(a.M);
  a.mtiles = (int)((a.M + NT - 1) / NT);
  int rb = 0;
  for (int p = 0; p < a.nprob; ++p) {
    a.p_rb0[p] = rb;
    rb += (a.p_out[p] + kUmRows - 1) / kUmRows;
  }
  a.p_rb0[a.nprob] = rb;
  a.row_blocks = rb;
  if ((int64_t)rb * a.mtiles < sm_count()) return -1;
  if (!encode_fn()) return -1;
  void* xh = ws;
  void* xl = lo ? static_cast<char*>(ws) + opnd : nullptr;
  int s = tc_operands(a0, xh, xl, val_dtype, st);
  if (s != VQ2_OK) return s;
  a.x = xh;
  a.x_row_stride = a.n;
  a.x_mode = VQ2_ACT_ROTATED;
  if (val_dtype == VQ2_F16) return res ? launch_umma_nt<true, __half>(a, xh, xl, st) : launch_umma_nt<false, __half>(a, xh, xl, st);
  return res ? launch_umma_nt<true, __nv_bfloat16>(a, xh, xl, st) : launch_umma_nt<false, __nv_bfloat16>(a, xh, xl, st);
}

}  // namespace vq2

extern "C" int vq2_tc_status(int reset) {
  int32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_umma_status, sizeof(v));
  if (e != cudaSuccess) {
    vq2::set_last_cuda_error(e);
    return VQ2_ERR_LAUNCH;
  }
  if (reset) {
    const int32_t z = 0;
    e = cudaMemcpyToSymbol(g_umma_status, &z, sizeof(z));
    if (e != cudaSuccess) {
      vq2::set_last_cuda_error(e);
      return VQ2_ERR_LAUNCH;
    }
  }
  return v;
}
