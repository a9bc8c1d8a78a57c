// Tensor-core Q4_0 GEMM for prompt prefill: Y[t][n] = bf16(sum_k W[n][k] X[t][k]).
//
// The reference's prefill multiplies the chunk's activations by the bf16 dequantization
// of each Q4_0 weight (integration/weights.py:28-31 `dequantize(...).bfloat16()`, then
// vLLM's torch matmul, integration/model.py:50-62).  This kernel computes the same
// product without a bf16 copy of the weights in HBM: the Q4_0 planes are dequantized
// straight into shared memory (w = bf16(fp32(d) * (q - 8)), the rounding of
// spark_q4_dequantize_bf16) and multiplied on the tensor cores (tcgen05.mma kind::f16,
// bf16 operands, fp32 accumulators in tensor memory).
//
// Persistent, warp-specialized; one CTA per SM walks output tiles of 128 weight rows
// (MMA M = TMEM lanes) x bn tokens (MMA N = TMEM columns; the host passes bn = 256, the
// kernel also takes 128).  448 threads:
//   warp 0      TMA producer: per 64-wide K step the activation tile X[bn][64] (bf16,
//               128-byte swizzle); per 256-wide K stage the weight rows' nibbles
//               [128][128 B] (128-byte swizzle) and fp16 scales [128][8];
//   warp 1      owns the tensor memory (512 columns: two accumulators, so the epilogue
//               of one tile overlaps the main loop of the next); one lane issues the
//               4 MMAs (K = 16 each) of every K step and the commits;
//   warps 2-9   dequantize: thread (row r, half h) writes block h of row r's K step as
//               32 bf16 into the 128-byte-swizzled K-major weight tile;
//   warps 10-13 epilogue: tcgen05.ld of their 32 TMEM lanes, bf16, stores to Y.
// Rings: X 4 stages, dequantized weights 3 stages, raw Q4_0 2 stages (213 KB).
//
// Both operand tiles are K-major with the 128-byte swizzle: row r of a tile at
// (r / 8) * 1024 + (r % 8) * 128, its 16-byte chunk c at chunk position c ^ (r % 8) --
// the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B and the MMA descriptors read.
//
// Every mbarrier wait is bounded by %globaltimer (limit_ns, a kernel argument).  A wait
// that runs out sets *error = 1 and a CTA-wide abort flag that every other wait checks,
// so all roles leave their loops.  Before the CTA frees anything, the producer waits
// (bound kDrainNs) for the bulk copies it issued and the MMA lane commits once more and
// waits (same bound) for that commit, which tracks every MMA it issued.  If that drain
// runs out, *error = 2 and the CTA exits WITHOUT freeing its tensor memory: the context
// must then be treated as unusable.  tcgen05.alloc itself has no bound: it blocks until
// 512 columns are free, so the kernel assumes no other tensor-memory user on the SM (its
// 213 KB of shared memory keeps it at one CTA per SM).
#pragma once

#include <cuda.h>

#include <cstdint>

#include "common.cuh"

namespace spark {
namespace tc {

constexpr int kBM = 128;        // weight rows per tile (MMA M)
constexpr int kBNMax = 256;     // tokens per tile (MMA N)
constexpr int kBK = 64;         // K per MMA step: one 128-byte swizzle atom of bf16
constexpr int kRK = 256;        // K per raw Q4_0 stage: 128 B of nibbles per row
constexpr int kStepsPerR = kRK / kBK;
constexpr int kXStages = 4, kAStages = 3, kRStages = 2;
constexpr int kXBytes = kBNMax * kBK * 2;      // 32 KB
constexpr int kABytes = kBM * kBK * 2;         // 16 KB
constexpr int kRQBytes = kBM * kRK / 2;        // 16 KB of nibbles
constexpr int kRDBytes = kBM * (kRK / 32) * 2;  // 2 KB of fp16 scales
constexpr int kOffX = 0;
constexpr int kOffA = kOffX + kXStages * kXBytes;
constexpr int kOffRQ = kOffA + kAStages * kABytes;
constexpr int kOffRD = kOffRQ + kRStages * kRQBytes;
constexpr int kOffBar = kOffRD + kRStages * kRDBytes;
// barriers: x_full, x_empty, a_full, a_empty, r_full, r_empty, t_full, t_empty, drain
constexpr int kBarXFull = 0, kBarXEmpty = kBarXFull + kXStages, kBarAFull = kBarXEmpty + kXStages,
              kBarAEmpty = kBarAFull + kAStages, kBarRFull = kBarAEmpty + kAStages,
              kBarREmpty = kBarRFull + kRStages, kBarTFull = kBarREmpty + kRStages, kBarTEmpty = kBarTFull + 2,
              kBarDrain = kBarTEmpty + 2, kNumBars = kBarDrain + 1;
constexpr int kOffMisc = kOffBar + 8 * kNumBars;  // tmem base, abort flag, drained flag
constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + 1024-B alignment slack
constexpr int kThreads = 448;
constexpr int kDeqWarp0 = 2, kDeqWarps = 8, kEpiWarp0 = 10;
constexpr int kTmemCols = 512;
constexpr unsigned long long kWaitNs = 500ull * 1000 * 1000;    // default limit of a wait: 0.5 s
constexpr unsigned long long kDrainNs = 2000ull * 1000 * 1000;  // drain of issued copies / MMAs

static_assert(kSmemBytes <= 227 * 1024, "shared memory");
static_assert(kOffA % 1024 == 0 && kOffRQ % 1024 == 0, "swizzled tiles need 1024-B alignment");

// instruction descriptor (kind::f16): fp32 D (bits 4-5 = 1), bf16 A (bits 7-9 = 1) and
// B (bits 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24
__host__ __device__ constexpr uint32_t idesc(int bn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// shared-memory matrix descriptor of a K-major 128-byte-swizzled tile at `addr`
// (1024-byte aligned): start >> 4, leading offset 16 B (unused with this swizzle),
// 8-row groups 1024 B apart, descriptor version 1, layout SWIZZLE_128B (2)
__device__ __forceinline__ uint64_t sdesc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase of `parity` to complete.  false: limit_ns ran out, or (abort given)
// another role set the abort flag.  A limit of 0 gives up after the second look.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, unsigned long long limit_ns,
                                         const volatile int* abort) {
  unsigned long long t0 = 0;
  for (;;) {
    uint32_t done;
    asm volatile(
        "{.reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p;}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (abort && *abort) return false;
    const unsigned long long t = now_ns();
    if (t0 == 0) t0 = t;
    else if (t - t0 >= limit_ns) return false;
  }
}

__device__ __forceinline__ void bar_init(uint32_t bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// 2-D tiled TMA load of this GPU's memory into this CTA's shared memory (no multicast)
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

// 8 weights of one Q4_0 block as 4 bf16 pairs: the nibbles at `shift` (0: low, 4: high)
// of the 8 bytes held by (w0, w1).  A byte permute puts each masked nibble byte b under
// the exponent of 2^23, giving fp32 2^23 + b exactly (b = q, or 16 q for the high
// nibbles); subtracting 2^23 + 8 (2^23 + 128) leaves q - 8 (16 (q - 8)) exactly, and the
// product with fp32(d) (d / 16) is exact in fp32 (11 + 4 significant bits).  The pairs go
// through packed f32x2 arithmetic, and cvt.rn.bf16x2 rounds each pair to nearest-even
// (NaN -> 0x7fff), the same bits as f2bf of fp32(d) * (q - 8) (a zero product may come out
// as +0 where that gives -0).  d finite.
__device__ __forceinline__ uint4 deq8(uint32_t w0, uint32_t w1, int shift, float s) {
  const uint32_t m = shift ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
  const float off = shift ? -8388736.0f : -8388616.0f;  // -(2^23 + 128), -(2^23 + 8)
  const float sc = shift ? s * 0.0625f : s;             // exact: a power-of-two scale
  const unsigned long long off2 = pack2(off, off), sc2 = pack2(sc, sc);
  const uint32_t a = w0 & m, b = w1 & m;
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t wd = i < 2 ? a : b;
    const uint32_t k = (2 * i) & 3;  // bytes k, k + 1 of the word: one bf16 pair
    const float f0 = __uint_as_float(__byte_perm(wd, 0x4B000000u, 0x7440u | k));
    const float f1 = __uint_as_float(__byte_perm(wd, 0x4B000000u, 0x7440u | (k + 1)));
    unsigned long long v = pack2(f0, f1);
    asm("add.rn.f32x2 %0, %0, %1;" : "+l"(v) : "l"(off2));
    asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(v) : "l"(sc2));
    float p0, p1;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(p0), "=f"(p1) : "l"(v));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(o[i]) : "f"(p1), "f"(p0));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

// Tensor maps (host-encoded): tmx over X [T][K] bf16, box {64, bn}, 128-byte swizzle;
// tmq over the nibble plane [N][K/2] bytes, box {128, 128}, 128-byte swizzle; tmd over
// the scale plane [N][K/32] fp16, box {8, 128}.  K % 256 == 0.
__global__ void __launch_bounds__(kThreads, 1)
    q4_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmq,
                      const __grid_constant__ CUtensorMap tmd, uint16_t* __restrict__ y, int T, int N, int K, int bn,
                      int* __restrict__ error, unsigned long long limit_ns) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = (uint32_t)__cvta_generic_to_shared(smem_raw);
  const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;
  const uint32_t base = raw + pad;
  unsigned char* gbase = smem_raw + pad;
  const uint32_t bars = base + kOffBar;
  const uint32_t tslot = base + kOffMisc;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + kOffMisc + 4);
  volatile int* drained_flag = reinterpret_cast<volatile int*>(gbase + kOffMisc + 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = K / kBK;
  const int ntn = (T + bn - 1) / bn, ntm = (N + kBM - 1) / kBM, ntiles = ntn * ntm;
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
  auto fail = [&]() {
    atomicCAS(error, 0, 1);
    *abort_flag = 1;
  };

  if (tid == 0) {
    for (int s = 0; s < kXStages; s++) {
      bar_init(bar(kBarXFull + s), 1);
      bar_init(bar(kBarXEmpty + s), 1);
    }
    for (int s = 0; s < kAStages; s++) {
      bar_init(bar(kBarAFull + s), kDeqWarps);
      bar_init(bar(kBarAEmpty + s), 1);
    }
    for (int s = 0; s < kRStages; s++) {
      bar_init(bar(kBarRFull + s), 1);
      bar_init(bar(kBarREmpty + s), kDeqWarps);
    }
    for (int s = 0; s < 2; s++) {
      bar_init(bar(kBarTFull + s), 1);
      bar_init(bar(kBarTEmpty + s), 4);
    }
    bar_init(bar(kBarDrain), 1);
    *abort_flag = 0;
    *drained_flag = 1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tslot), "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  uint32_t tmem;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(tmem) : "r"(tslot) : "memory");

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t ix = 0, ir = 0;  // copies issued
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int mt = tile / ntn, nt = tile - mt * ntn;
        for (int kb = 0; kb < nk; kb++) {
          if (kb % kStepsPerR == 0) {
            const uint32_t s = ir % kRStages;
            if (!bar_wait(bar(kBarREmpty + s), ((ir / kRStages) & 1) ^ 1, limit_ns, abort_flag)) {
              ok = false;
              break;
            }
            bar_expect_tx(bar(kBarRFull + s), kRQBytes + kRDBytes);
            tma_load_2d(base + kOffRQ + s * kRQBytes, &tmq, (kb / kStepsPerR) * (kRK / 2), mt * kBM,
                        bar(kBarRFull + s));
            tma_load_2d(base + kOffRD + s * kRDBytes, &tmd, (kb / kStepsPerR) * (kRK / 32), mt * kBM,
                        bar(kBarRFull + s));
            ir++;
          }
          const uint32_t s = ix % kXStages;
          if (!bar_wait(bar(kBarXEmpty + s), ((ix / kXStages) & 1) ^ 1, limit_ns, abort_flag)) {
            ok = false;
            break;
          }
          bar_expect_tx(bar(kBarXFull + s), (uint32_t)bn * kBK * 2);
          tma_load_2d(base + kOffX + s * kXBytes, &tmx, kb * kBK, nt * bn, bar(kBarXFull + s));
          ix++;
        }
      }
      if (!ok) fail();
      // every issued copy lands before the CTA can give its shared memory up
      bool drained = true;
      for (uint32_t i = ix > (uint32_t)kXStages ? ix - kXStages : 0; i < ix; i++)
        drained &= bar_wait(bar(kBarXFull + i % kXStages), (i / kXStages) & 1, kDrainNs, nullptr);
      for (uint32_t i = ir > (uint32_t)kRStages ? ir - kRStages : 0; i < ir; i++)
        drained &= bar_wait(bar(kBarRFull + i % kRStages), (i / kRStages) & 1, kDrainNs, nullptr);
      if (!drained) {
        atomicExch(error, 2);
        *drained_flag = 0;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t ix = 0, ia = 0, ti = 0;
      bool ok = true;
      const uint32_t id = idesc(bn);
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ti++) {
        const uint32_t acc = ti & 1;
        if (!bar_wait(bar(kBarTEmpty + acc), ((ti >> 1) & 1) ^ 1, limit_ns, abort_flag)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t dt = tmem + acc * kBNMax;
        for (int kb = 0; kb < nk; kb++) {
          const uint32_t sx = ix % kXStages, sa = ia % kAStages;
          if (!bar_wait(bar(kBarXFull + sx), (ix / kXStages) & 1, limit_ns, abort_flag) ||
              !bar_wait(bar(kBarAFull + sa), (ia / kAStages) & 1, limit_ns, abort_flag)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t ad = sdesc(base + kOffA + sa * kABytes), bd = sdesc(base + kOffX + sx * kXBytes);
#pragma unroll
          for (int j = 0; j < kBK / 16; j++) {  // K = 16 per MMA: 32 bytes further along the swizzled rows
            const uint32_t accum = (kb | j) != 0;
            asm volatile(
                "{.reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;}" ::"r"(
                    dt),
                "l"(ad + 2 * j), "l"(bd + 2 * j), "r"(id), "r"(accum));
          }
          mma_commit(bar(kBarXEmpty + sx));
          mma_commit(bar(kBarAEmpty + sa));
          ix++;
          ia++;
        }
        if (!ok) break;
        mma_commit(bar(kBarTFull + acc));
      }
      if (!ok) fail();
      // the drain commit tracks every MMA issued before it
      mma_commit(bar(kBarDrain));
      if (!bar_wait(bar(kBarDrain), 0, kDrainNs, nullptr)) {
        atomicExch(error, 2);
        *drained_flag = 0;
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ---------------------------------------------------------------- dequantize
    const int u = tid - 32 * kDeqWarp0;
    const int r = u & (kBM - 1), h = u >> 7;  // row r of the tile, block h of each K step
    uint32_t ir = 0, ia = 0;
    bool ok = true;
    uint4 sc = make_uint4(0, 0, 0, 0);
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < nk; kb++) {
        const uint32_t rs = ir % kRStages;
        if (kb % kStepsPerR == 0) {
          ok = __all_sync(0xffffffffu, bar_wait(bar(kBarRFull + rs), (ir / kRStages) & 1, limit_ns, abort_flag));
          if (!ok) break;
          sc = lds128(base + kOffRD + rs * kRDBytes + r * 16);  // the row's 8 block scales
        }
        const uint32_t sa = ia % kAStages;
        ok = __all_sync(0xffffffffu, bar_wait(bar(kBarAEmpty + sa), ((ia / kAStages) & 1) ^ 1, limit_ns, abort_flag));
        if (!ok) break;
        const int j = kb % kStepsPerR, blk = 2 * j + h;
        const uint4 q = lds128(base + kOffRQ + rs * kRQBytes + r * 128 + ((blk ^ (r & 7)) << 4));
        const uint32_t sw = blk < 4 ? (blk < 2 ? sc.x : sc.y) : (blk < 6 ? sc.z : sc.w);
        const float s = h2f((uint16_t)((blk & 1) ? (sw >> 16) : (sw & 0xffffu)));
        const uint32_t a = base + kOffA + sa * kABytes;
        sts128(a + sw128(r, 4 * h + 0), deq8(q.x, q.y, 0, s));
        sts128(a + sw128(r, 4 * h + 1), deq8(q.z, q.w, 0, s));
        sts128(a + sw128(r, 4 * h + 2), deq8(q.x, q.y, 4, s));
        sts128(a + sw128(r, 4 * h + 3), deq8(q.z, q.w, 4, s));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) bar_arrive(bar(kBarAFull + sa));
        ia++;
        if (j == kStepsPerR - 1) {  // the stage's last K step: its raw bytes are free
          if (lane == 0) bar_arrive(bar(kBarREmpty + rs));
          ir++;
        }
      }
    }
    if (!ok) fail();
  } else {
    // ---------------------------------------------------------------- epilogue
    const int qd = warp & 3;  // TMEM lanes 32 qd .. 32 qd + 31
    uint32_t ti = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ti++) {
      const int mt = tile / ntn, nt = tile - mt * ntn;
      const uint32_t acc = ti & 1;
      ok = __all_sync(0xffffffffu, bar_wait(bar(kBarTFull + acc), (ti >> 1) & 1, limit_ns, abort_flag));
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int row = mt * kBM + qd * 32 + lane;
      const int tok0 = nt * bn;
#pragma unroll 1
      for (int c0 = 0; c0 < bn; c0 += 16) {
        uint32_t v[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(tmem + ((uint32_t)(qd * 32) << 16) + acc * kBNMax + (uint32_t)c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;"
                     : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]),
                       "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]),
                       "+r"(v[14]), "+r"(v[15])
                     :
                     : "memory");
        if (row < N) {
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int tt = tok0 + c0 + i;
            if (tt < T) y[(size_t)tt * N + row] = f2bf(__uint_as_float(v[i]));
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) bar_arrive(bar(kBarTEmpty + acc));
    }
    if (!ok) fail();
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1 && *drained_flag) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

}  // namespace tc
}  // namespace spark
