// tcgen05 projection GEMMs for the Hyena mixer (sm_100a).
//
//   in_proj : out(M,N) bf16 = (A e4m3 . B e4m3^T) * sa * sb     (kind::f8f6f4)
//   out_proj: out(M,N) bf16 =  A bf16 . B bf16^T + bias          (kind::f16)
// Both operands K-major (activations (M,K) row-major, nn.Linear weights (N,K)).
//
// Persistent kernel, one CTA per SM, walking 128 x BN output tiles (N fastest)
// with two fp32 accumulators in tensor memory so that a tile's epilogue overlaps
// the next tile's main loop:
//   warp 0     TMA producer: 128-byte-wide K slabs of A and B, SWIZZLE_128B,
//              into a multi-stage shared-memory ring (no multicast)
//   warp 1     TMEM allocation + single-thread tcgen05.mma issue; each stage is
//              released by tcgen05.commit onto its "empty" mbarrier, each
//              finished accumulator by a commit onto its "acc_full" mbarrier
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time, scale / bias, bf16,
//              16-byte global stores; the accumulator is handed back ("acc_empty")
//              as soon as its last column is in registers
// Small M (decode batches) cannot fill the SMs with output tiles, so K is split
// across the CTAs of a thread-block cluster instead (gemm_cluster_kernel): each
// CTA accumulates its K slice in TMEM, parks the fp32 partial in its own shared
// memory, and after a cluster barrier every CTA sums a row slice of all the
// partials over DSMEM in a fixed order (deterministic; no workspace, no atomics,
// no second launch).
// Every mbarrier wait is bounded by a globaltimer budget; on expiry the kernel
// records the event in a device counter and runs to completion (TMEM freed);
// hyena_gemm_wait_timeouts reads the counter back, so a GEMM that gave up
// (and wrote an incomplete tile) is reported instead of passing silently.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "common.cuh"

namespace hb {
namespace gemm {

constexpr int BM = 128;
constexpr int BKB = 128;  // bytes of K per stage (one 128B swizzle row)
constexpr int THREADS = 192;
constexpr unsigned long long WAIT_BUDGET_NS = 4000000000ull;  // 4 s

// Tile configuration for an N-tile of BN columns: as many pipeline stages as
// fit in ~192 KB of shared memory (4 at BN = 256, 8 at BN <= 64), and a TMEM
// accumulator of BN fp32 columns.
template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BKB;
  static constexpr int B_BYTES = BN * BKB;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024 / STAGE_BYTES) > 8 ? 8 : (192 * 1024 / STAGE_BYTES);
  // two accumulators, allocated as a power of two >= 32 columns (BN = 192: 512)
  static constexpr uint32_t TMEM_COLS =
      2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
};

template <int BN>
struct __align__(1024) Smem {
  uint8_t a[Cfg<BN>::STAGES][Cfg<BN>::A_BYTES];
  uint8_t b[Cfg<BN>::STAGES][Cfg<BN>::B_BYTES];
  uint64_t full[Cfg<BN>::STAGES];
  uint64_t empty[Cfg<BN>::STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
};

__device__ int g_wait_timeouts;

__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of `parity` to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
  if (mbar_try_wait(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  while (true) {
    if (mbar_try_wait(b, parity)) return true;
    if (now_ns() - t0 > WAIT_BUDGET_NS) {
      atomicAdd(&g_wait_timeouts, 1);
      return false;
    }
  }
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
// TMA tile load with an L2 eviction-priority hint (createpolicy).
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(su32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// Tile of a tensor map into L2 only (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 16-byte store marked streaming (evict-first in L2): GEMM outputs are read
// once, later, by another kernel, and must not push the weights out of L2.
__device__ __forceinline__ void st_stream16(void* p, const uint4& v) {
  asm volatile("st.global.cs.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// K-major, SWIZZLE_128B shared-memory matrix descriptor: 8-row core groups
// 1024 B apart (SBO), LBO unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
  const uint64_t addr = su32(p);
  return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}
template <bool FP8>
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                    uint32_t accumulate) {
  if constexpr (FP8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
  }
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          su32(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The same load without the wait, so that several can be in flight.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Instruction descriptor: fp32 accumulator, K-major A and B, M=128, N=256;
// operand format E4M3 (kind::f8f6f4) or BF16 (kind::f16).
template <bool FP8, int BN>
__host__ __device__ constexpr uint32_t idesc() {
  return (1u << 4) | ((FP8 ? 0u : 1u) << 7) | ((FP8 ? 0u : 1u) << 10) |
         (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}

template <bool FP8, int BN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            bf16* __restrict__ out, int64_t ldo, int M, int N, int K,
            const float* __restrict__ sa, const float* __restrict__ sb,
            const bf16* __restrict__ bias) {
  constexpr int STAGES = Cfg<BN>::STAGES;
  constexpr int STAGE_BYTES = Cfg<BN>::STAGE_BYTES;
  constexpr uint32_t TMEM_COLS = Cfg<BN>::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  Smem<BN>& S = *reinterpret_cast<Smem<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr int ELEM = FP8 ? 1 : 2;
  constexpr int KE = BKB / ELEM;  // K elements per stage
  const int kblocks = K / KE;
  // Tiles in N-fastest order: CTAs resident together share A row panels, and the
  // whole weight (<= 50 MB at the 7B shape) stays in L2 while the activations
  // stream through once.
  const int n_tiles = (N + BN - 1) / BN;
  const int total = n_tiles * ((M + BM - 1) / BM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.acc_full[b], 1);
      mbar_init(&S.acc_empty[b], 4);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(&S.tmem_base)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = S.tmem_base;
  // While the previous kernel drains: this CTA's first weight tiles into L2
  // (a prefetch cannot observe stale data: L2 is the point of coherence).
  if (warp == 0 && lane == 0 && (int)blockIdx.x < total) {
    const int n0 = ((int)blockIdx.x % n_tiles) * BN;
    for (int kb = 0; kb < kblocks && kb < STAGES; ++kb) tma_prefetch_l2(&tmB, kb * KE, n0);
  }
  pdl_wait();
  pdl_trigger();  // after the wait: see common.cuh

  if (warp == 0) {
    if (lane == 0) {
      // Many M tiles (prefill): the weight panel is reused by every M tile, the
      // activations once per N tile -> keep B, stream A.  Few M tiles (decode):
      // A is reused by every N tile, the weight streamed once per call.
      const bool many_m = (M + BM - 1) / BM > 8;
      const uint64_t pol_a = many_m ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_b = many_m ? policy_evict_last() : policy_evict_first();
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&S.empty[s], ((it / STAGES) & 1) ^ 1)) { ok = false; break; }
          mbar_expect_tx(&S.full[s], STAGE_BYTES);
          tma_load_2d(&tmA, &S.full[s], S.a[s], kb * KE, m0, pol_a);
          tma_load_2d(&tmB, &S.full[s], S.b[s], kb * KE, n0, pol_b);
        }
      }
      // Drain: every issued copy has landed before the CTA can exit.
      for (uint32_t i = it > (uint32_t)STAGES ? it - STAGES : 0; i < it; ++i)
        mbar_wait(&S.full[i % STAGES], (i / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID = idesc<FP8, BN>();
      uint32_t it = 0, ti = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++ti) {
        const int b = ti & 1;
        if (!mbar_wait(&S.acc_empty[b], ((ti >> 1) & 1) ^ 1)) ok = false;
        fence_after();
        const uint32_t d = tmem + uint32_t(b * BN);
        for (int kb = 0; kb < kblocks && ok; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&S.full[s], (it / STAGES) & 1)) { ok = false; break; }
          fence_after();
#pragma unroll
          for (int kk = 0; kk < BKB / 32; ++kk) {
            const uint64_t ad = sw128_desc(S.a[s] + kk * 32);
            const uint64_t bd = sw128_desc(S.b[s] + kk * 32);
            mma<FP8>(d, ad, bd, ID, (kb != 0 || kk != 0) ? 1u : 0u);
          }
          mma_commit(&S.empty[s]);
        }
        mma_commit(&S.acc_full[b]);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    float scale_a = 1.0f, scale_b = 1.0f;
    if constexpr (FP8) {
      scale_a = __ldg(sa);
      scale_b = __ldg(sb);
    }
    uint32_t ti = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++ti) {
      const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
      const int b = ti & 1;
      const bool ok = mbar_wait(&S.acc_full[b], (ti >> 1) & 1);
      if (!ok) break;  // the MMA warp gave up: stop rather than time out per tile
      fence_after();
      const int row = m0 + 32 * q + lane;
#pragma unroll 1
      for (int cb = 0; cb < BN / 32; ++cb) {
        uint32_t r[32];
        tmem_ld32(tmem + (uint32_t(32 * q) << 16) + uint32_t(b * BN + cb * 32), r);
        if (cb == BN / 32 - 1) {  // accumulator fully read: hand it back to the MMA warp
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.acc_empty[b]);
        }
        const int col0 = n0 + cb * 32;
        if (row >= M || col0 >= N) continue;
        bf16* dst = out + (long long)row * ldo + col0;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          if (col0 + 8 * v >= N) break;
          uint4 pk;
          uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float x0 = __uint_as_float(r[8 * v + 2 * e]);
            float x1 = __uint_as_float(r[8 * v + 2 * e + 1]);
            if constexpr (FP8) {
              x0 = (x0 * scale_a) * scale_b;  // (acc * sx) * sw, fp8_emul.py:87
              x1 = (x1 * scale_a) * scale_b;
            } else {
              if (bias != nullptr) {
                x0 += __bfloat162float(bias[col0 + 8 * v + 2 * e]);
                x1 += __bfloat162float(bias[col0 + 8 * v + 2 * e + 1]);
              }
            }
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
            pw[e] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          st_stream16(dst + 8 * v, pk);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------- small M
// Shared memory of the cluster split-K kernel.  After the main loop the ring
// is reused as
//   staging  [BM][LD]            this CTA's fp32 partial, rows other CTAs own
//   inbox    [splits-1][R][LD]   the other ranks' partials of the rows this CTA
//                                owns (slots in rank order, skipping itself)
// with R = ceil(BM / splits) and rows padded to LD = BN + 4 floats, so that a
// warp's 16-byte accesses to 32 consecutive rows fall in distinct banks.
template <int BN>
__host__ __device__ constexpr int max_cluster_splits() {
  return BN >= 256 ? 3 : 4;
}
constexpr int max_inbox_rows(int ms) {  // max over splits 2..ms of (splits-1) ceil(BM/splits)
  int best = 0;
  for (int sp = 2; sp <= ms; ++sp) {
    const int r = (sp - 1) * ((BM + sp - 1) / sp);
    best = r > best ? r : best;
  }
  return best;
}
template <int BN>
struct __align__(1024) SmemSK {
  static constexpr int RED_LD = BN + 4;
  static constexpr int INBOX_ROWS = max_inbox_rows(max_cluster_splits<BN>());
  static constexpr int RED_ROWS = BM + INBOX_ROWS;
  union {
    struct {
      uint8_t a[Cfg<BN>::STAGES][Cfg<BN>::A_BYTES];
      uint8_t b[Cfg<BN>::STAGES][Cfg<BN>::B_BYTES];
    } ring;
    float red[RED_ROWS * RED_LD];
  } u;
  uint64_t full[Cfg<BN>::STAGES];
  uint64_t empty[Cfg<BN>::STAGES];
  uint64_t acc_full;
  uint64_t inbox_full;
  float bias_s[BN];
  uint32_t tmem_base;
};

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Bulk copy of `bytes` from this CTA's shared memory into another CTA's
// (cluster address), completing `bytes` of transaction count on that CTA's
// mbarrier (cluster address).
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst, uint32_t src, uint32_t bytes,
                                                     uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst), "r"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
template <int N>
__host__ __device__ constexpr uint32_t pow2_cols() {
  return N <= 32 ? 32u : N <= 64 ? 64u : N <= 128 ? 128u : N <= 256 ? 256u : 512u;
}

// One 128 x BN output tile per cluster of `splits` CTAs (grid (splits, tiles),
// cluster (splits, 1, 1); splits = 1 is a plain one-tile-per-CTA GEMM).  CTA r
// accumulates K blocks [r kblocks / splits, (r+1) kblocks / splits) in TMEM and
// owns rows [r R, (r+1) R) of the tile.  Each CTA stages its whole fp32
// partial tile in its own (idle) ring; once every CTA of the cluster has
// finished its main loop (split arrive / wait cluster barrier, the staging in
// between), each epilogue warp sends its rows to their owners with one bulk
// copy per owner; every owner waits for its inbox on an mbarrier and all six
// warps sum the ranks' partials in rank order (deterministic), scale / add
// bias and store bf16 rows coalesced.  A second split barrier (arrive once the
// inbox is full, wait before exit) keeps every staging area alive until all
// copies have landed.
template <bool FP8, int BN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_cluster_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, bf16* __restrict__ out, int64_t ldo,
                    int M, int N, int K, const float* __restrict__ sa,
                    const float* __restrict__ sb, const bf16* __restrict__ bias) {
  constexpr int STAGES = Cfg<BN>::STAGES;
  constexpr int STAGE_BYTES = Cfg<BN>::STAGE_BYTES;
  constexpr uint32_t TMEM_COLS = pow2_cols<BN>();
  constexpr int LD = SmemSK<BN>::RED_LD;
  static_assert(BN % 32 == 0, "epilogue reads 32 columns at a time");
  extern __shared__ uint8_t smem_raw[];
  SmemSK<BN>& S = *reinterpret_cast<SmemSK<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                 ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr int ELEM = FP8 ? 1 : 2;
  constexpr int KE = BKB / ELEM;
  const int kblocks = K / KE;
  const int splits = (int)gridDim.x;
  const int rank = (int)cluster_rank();
  const int rows_per = (BM + splits - 1) / splits;
  const int n_tiles = (N + BN - 1) / BN;
  const int tile = (int)blockIdx.y;
  const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
  const int kb0 = rank * kblocks / splits, kb1 = (rank + 1) * kblocks / splits;
  const int rows = M - m0 < BM ? M - m0 : BM;  // valid rows of the tile
  // Rows [o R, o R + owned(o)) belong to rank o.
  auto owned = [&](int o) {
    const int lo = o * rows_per, hi = (o + 1) * rows_per < rows ? (o + 1) * rows_per : rows;
    return hi > lo ? hi - lo : 0;
  };
  const int my_rows = owned(rank);
  const uint32_t inbox_bytes = uint32_t((splits - 1) * my_rows * LD * 4);
  float* staging = S.u.red;
  float* inbox = S.u.red + BM * LD;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    mbar_init(&S.acc_full, 1);
    mbar_init(&S.inbox_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(&S.inbox_full, inbox_bytes);  // the one arrival; the copies bring the bytes
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(&S.tmem_base)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = S.tmem_base;
  // While the previous kernel drains: this CTA's first weight tiles into L2.
  if (warp == 0 && lane == 0) {
    for (int kb = kb0; kb < kb1 && kb < kb0 + STAGES; ++kb) tma_prefetch_l2(&tmB, kb * KE, n0);
  }
  pdl_wait();
  pdl_trigger();  // after the wait: see common.cuh

  if (warp == 0) {
    if (lane == 0) {
      // The activations are re-read by every tile's cluster, the weights once.
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_evict_first();
      int it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&S.empty[s], ((it / STAGES) & 1) ^ 1)) break;
        mbar_expect_tx(&S.full[s], STAGE_BYTES);
        tma_load_2d(&tmA, &S.full[s], S.u.ring.a[s], kb * KE, m0, pol_a);
        tma_load_2d(&tmB, &S.full[s], S.u.ring.b[s], kb * KE, n0, pol_b);
      }
      // Drain: every issued copy has landed before the ring is reused.
      for (int i = it > STAGES ? it - STAGES : 0; i < it; ++i)
        mbar_wait(&S.full[i % STAGES], (i / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID = idesc<FP8, BN>();
      int it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&S.full[s], (it / STAGES) & 1)) break;
        fence_after();
#pragma unroll
        for (int kk = 0; kk < BKB / 32; ++kk) {
          const uint64_t ad = sw128_desc(S.u.ring.a[s] + kk * 32);
          const uint64_t bd = sw128_desc(S.u.ring.b[s] + kk * 32);
          mma<FP8>(tmem, ad, bd, ID, (kb != kb0 || kk != 0) ? 1u : 0u);
        }
        mma_commit(&S.empty[s]);
      }
      mma_commit(&S.acc_full);  // fires once every MMA above has completed
    }
  }
  bool have = false;
  float scale = 1.0f, scale_b = 1.0f;
  if constexpr (FP8) {  // every warp takes part in the final reduction
    scale = __ldg(sa);
    scale_b = __ldg(sb);
  }
  if (warp >= 2) {
    // While the main loop runs: epilogue constants into registers / shared memory.
    if constexpr (!FP8) {
      for (int j = threadIdx.x - 64; j < BN; j += 128)
        S.bias_s[j] = (bias != nullptr && n0 + j < N) ? __bfloat162float(bias[n0 + j]) : 0.0f;
    }
    have = __all_sync(0xffffffffu, kb1 > kb0 && mbar_wait(&S.acc_full, 0));
  }
  // Barrier 1 (split arrive / wait): once every CTA of the cluster has arrived
  // its main loop is over (producer drained, accumulator complete), so every
  // ring may be staging / inbox.  Each CTA stages into its own ring between
  // its arrive and its wait.
  fence_before();
  __syncwarp();
  cluster_arrive();

  if (warp >= 2) {
    const int q = warp & 3;  // TMEM lane quarter of this epilogue warp
    const int row = 32 * q + lane;
    // Stage every row of the partial tile as fp32 (an empty K slice stages
    // zeros): the rows other ranks own go out by bulk copy, this rank's own
    // rows are summed from here with the inbox.
    if (__any_sync(0xffffffffu, row < rows)) {  // warp-uniform: TMEM loads are .sync.aligned
      float4* dst = reinterpret_cast<float4*>(staging + row * LD);
#pragma unroll 1
      for (int cb = 0; cb < BN / 32; cb += 2) {
        uint32_t r[2][32];
        if (have) {
          tmem_ld32_async(tmem + (uint32_t(32 * q) << 16) + uint32_t(cb * 32), r[0]);
          tmem_ld32_async(tmem + (uint32_t(32 * q) << 16) + uint32_t(cb * 32 + 32), r[1]);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[0][j] = r[1][j] = 0u;
        }
        if (row < rows) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[(cb + h) * 8 + v] =
                  make_float4(__uint_as_float(r[h][4 * v]), __uint_as_float(r[h][4 * v + 1]),
                              __uint_as_float(r[h][4 * v + 2]), __uint_as_float(r[h][4 * v + 3]));
        }
      }
    }
    fence_proxy_async_smem();  // this warp's staged rows -> visible to the bulk-copy engine
    __syncwarp();
    cluster_wait();  // barrier 1: every peer's ring is free for its inbox
    fence_after();
    // This warp's rows to their owners: one bulk copy per row, issued by the
    // row's lane, so that 32 copies per warp are in flight at once.
    {
      const int o = row / rows_per;
      if (row < rows && o != rank) {
        const int slot = rank < o ? rank : rank - 1;
        const uint32_t dst =
            map_to_rank(su32(inbox + (slot * rows_per + row - o * rows_per) * LD), (uint32_t)o);
        const uint32_t bar = map_to_rank(su32(&S.inbox_full), (uint32_t)o);
        bulk_copy_to_cluster(dst, su32(staging + row * LD), uint32_t(LD * 4), bar);
      }
    }
  } else {
    __syncwarp();
    cluster_wait();  // barrier 1
  }
  // Barrier 2 arrive: every copy into this CTA has landed (the wait at the end
  // keeps each CTA alive until its own outgoing copies have landed too).
  const bool ready = inbox_bytes == 0 || mbar_wait(&S.inbox_full, 0);
  __syncwarp();
  cluster_arrive_relaxed();  // orders nothing: the inbox mbarrier already did
  // Owned rows, by all warps, 4 columns per item and U items in flight per
  // thread: the ranks' partials summed in rank order (deterministic), scaled /
  // bias added, 4 bf16 stored (consecutive threads: consecutive 16-byte float4
  // reads, conflict-free, and consecutive 8-byte pieces of a row).
  if (__syncthreads_and(ready ? 1 : 0)) {
    constexpr int CPR = BN / 4;  // 4-column pieces per row
    constexpr int U = 8;
    constexpr int MAXS = max_cluster_splits<BN>();
    const int n_items = my_rows * CPR;
    const int base = rank * rows_per;
#pragma unroll 1
    for (int i0 = (int)threadIdx.x; i0 < n_items; i0 += U * THREADS) {
      float4 acc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int p = 0; p < MAXS; ++p) {  // unrolled: every partial's loads in flight together
        if (p >= splits) break;
        const float* pb = p == rank ? staging + base * LD
                                    : inbox + (p < rank ? p : p - 1) * rows_per * LD;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int it = i0 + u * THREADS;
          if (it < n_items) {
            const float4 x =
                *reinterpret_cast<const float4*>(pb + (it / CPR) * LD + (it % CPR) * 4);
            acc[u].x += x.x;
            acc[u].y += x.y;
            acc[u].z += x.z;
            acc[u].w += x.w;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int it = i0 + u * THREADS;
        if (it >= n_items) continue;
        const int lr = it / CPR, c = (it % CPR) * 4;
        float v[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if constexpr (FP8) {
            v[e] = (v[e] * scale) * scale_b;  // (acc * sx) * sw, fp8_emul.py:87
          } else {
            v[e] += S.bias_s[c + e];
          }
        }
        if (n0 + c < N) {
          const __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]);
          const __nv_bfloat162 h1 = __floats2bfloat162_rn(v[2], v[3]);
          uint2 pk;
          pk.x = *reinterpret_cast<const uint32_t*>(&h0);
          pk.y = *reinterpret_cast<const uint32_t*>(&h1);
          *reinterpret_cast<uint2*>(out + (long long)(m0 + base + lr) * ldo + n0 + c) = pk;
        }
      }
    }
  }
  // Barrier 2 wait: every owner has its inbox, so no staging area is still
  // being read when its CTA exits; every TMEM read above is done.
  cluster_wait();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------- 2-SM tiles
// Large M: a cluster of two CTAs (an SM pair) computes 256 x 256 output tiles
// with tcgen05.mma.cta_group::2.  CTA r of the pair stages rows [128 r, 128 r +
// 128) of the A slab and rows [128 r, 128 r + 128) of the B slab (weight rows,
// i.e. output columns) in its own ring; the MMA, issued by the even CTA, reads
// both CTAs' stages at the same offsets and leaves each CTA's 128 output rows x
// 256 columns in that CTA's tensor memory.  Per CTA and 128-byte K slab that is
// 32 KB of operands for a 128 x 256 product (48 KB with a 1-SM tile of the same
// size), so L2 serves a third less and six stages fit instead of four.
//   warp 0 (both CTAs)  TMA of the CTA's halves; every copy completes on the
//                       even CTA's "full" barrier, which expects both halves
//   warp 1 (even CTA)   MMA issue; a stage is released by a commit multicast to
//                       both CTAs' "empty" barriers, an accumulator by one to
//                       both CTAs' "acc_full"
//   warps 2-5           epilogue of the CTA's 128 rows; the accumulator goes back
//                       by arrivals (4 per CTA) on the even CTA's "acc_empty"
// Tensor memory is allocated pair-wise (cta_group::2, 2 x 256 columns).
constexpr int BN2 = 256;
struct Cfg2 {
  static constexpr int A_BYTES = BM * BKB;
  static constexpr int B_BYTES = (BN2 / 2) * BKB;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 6;
  static constexpr uint32_t TMEM_COLS = 2 * BN2;
};
struct __align__(1024) Smem2 {
  uint8_t a[Cfg2::STAGES][Cfg2::A_BYTES];
  uint8_t b[Cfg2::STAGES][Cfg2::B_BYTES];
  uint64_t full[Cfg2::STAGES];
  uint64_t empty[Cfg2::STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
};

// TMA tile load by either CTA of a pair, completing on the mbarrier at cluster
// address `bar` (the even CTA's).
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar, void* dst,
                                                 int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
template <bool FP8>
__device__ __forceinline__ void mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  if constexpr (FP8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
  }
}
// Arrive (once) on the mbarrier at the same offset in both CTAs of the pair
// when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  const uint16_t both = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(su32(bar)),
      "h"(both)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

template <bool FP8>
__host__ __device__ constexpr uint32_t idesc_pair() {
  return (1u << 4) | ((FP8 ? 0u : 1u) << 7) | ((FP8 ? 0u : 1u) << 10) |
         (uint32_t(BN2 >> 3) << 17) | (uint32_t((2 * BM) >> 4) << 24);
}

template <bool FP8>
__global__ void __launch_bounds__(THREADS, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 bf16* __restrict__ out, int64_t ldo, int M, int N, int K,
                 const float* __restrict__ sa, const float* __restrict__ sb,
                 const bf16* __restrict__ bias) {
  pdl_trigger();
  constexpr int STAGES = Cfg2::STAGES;
  extern __shared__ uint8_t smem_raw[];
  Smem2& S = *reinterpret_cast<Smem2*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr int ELEM = FP8 ? 1 : 2;
  constexpr int KE = BKB / ELEM;
  const int kblocks = K / KE;
  const uint32_t rank = cluster_rank();  // 0: the MMA-issuing CTA
  const int pair = (int)blockIdx.x / 2, npairs = (int)gridDim.x / 2;
  const int n_tiles = (N + BN2 - 1) / BN2;
  const int total = n_tiles * ((M + 2 * BM - 1) / (2 * BM));

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.acc_full[b], 1);
      mbar_init(&S.acc_empty[b], 8);  // 4 epilogue warps in each CTA of the pair
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(&S.tmem_base)),
                 "r"(Cfg2::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  // both CTAs' barriers exist before any copy or arrival can target them
  cluster_arrive();
  cluster_wait();
  fence_after();
  const uint32_t tmem = S.tmem_base;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      const bool many_m = (M + BM - 1) / BM > 8;
      const uint64_t pol_a = many_m ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_b = many_m ? policy_evict_last() : policy_evict_first();
      const uint32_t full0 = map_to_rank(su32(&S.full[0]), 0);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < total && ok; tile += npairs) {
        const int m0 = (tile / n_tiles) * 2 * BM + (int)rank * BM;
        const int n0 = (tile % n_tiles) * BN2 + (int)rank * (BN2 / 2);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&S.empty[s], ((it / STAGES) & 1) ^ 1)) { ok = false; break; }
          if (rank == 0) mbar_expect_tx(&S.full[s], 2 * Cfg2::STAGE_BYTES);
          const uint32_t bar = full0 + uint32_t(s * sizeof(uint64_t));
          tma_load_2d_pair(&tmA, bar, S.a[s], kb * KE, m0, pol_a);
          tma_load_2d_pair(&tmB, bar, S.b[s], kb * KE, n0, pol_b);
        }
      }
      // Drain: every issued copy has landed before the CTA can exit.  The
      // even CTA sees its "full" phases complete; the odd CTA sees the MMA
      // release the stages its copies filled.
      for (uint32_t i = it > (uint32_t)STAGES ? it - STAGES : 0; i < it; ++i) {
        if (rank == 0)
          mbar_wait(&S.full[i % STAGES], (i / STAGES) & 1);
        else
          mbar_wait(&S.empty[i % STAGES], (i / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      constexpr uint32_t ID = idesc_pair<FP8>();
      uint32_t it = 0, ti = 0;
      bool ok = true;
      for (int tile = pair; tile < total && ok; tile += npairs, ++ti) {
        const int b = ti & 1;
        if (!mbar_wait(&S.acc_empty[b], ((ti >> 1) & 1) ^ 1)) ok = false;
        fence_after();
        const uint32_t d = tmem + uint32_t(b * BN2);
        for (int kb = 0; kb < kblocks && ok; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&S.full[s], (it / STAGES) & 1)) { ok = false; break; }
          fence_after();
#pragma unroll
          for (int kk = 0; kk < BKB / 32; ++kk) {
            const uint64_t ad = sw128_desc(S.a[s] + kk * 32);
            const uint64_t bd = sw128_desc(S.b[s] + kk * 32);
            mma_pair<FP8>(d, ad, bd, ID, (kb != 0 || kk != 0) ? 1u : 0u);
          }
          mma_commit_pair(&S.empty[s]);
        }
        mma_commit_pair(&S.acc_full[b]);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    float scale_a = 1.0f, scale_b = 1.0f;
    if constexpr (FP8) {
      scale_a = __ldg(sa);
      scale_b = __ldg(sb);
    }
    const uint32_t acc_empty0 = map_to_rank(su32(&S.acc_empty[0]), 0);
    uint32_t ti = 0;
    for (int tile = pair; tile < total; tile += npairs, ++ti) {
      const int m0 = (tile / n_tiles) * 2 * BM + (int)rank * BM, n0 = (tile % n_tiles) * BN2;
      const int b = ti & 1;
      const bool ok = mbar_wait(&S.acc_full[b], (ti >> 1) & 1);
      if (!ok) break;  // the MMA warp gave up: stop rather than time out per tile
      fence_after();
      const int row = m0 + 32 * q + lane;
#pragma unroll 1
      for (int cb = 0; cb < BN2 / 32; ++cb) {
        uint32_t r[32];
        tmem_ld32(tmem + (uint32_t(32 * q) << 16) + uint32_t(b * BN2 + cb * 32), r);
        if (cb == BN2 / 32 - 1) {  // accumulator fully read: hand it back to the MMA warp
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc_empty0 + uint32_t(b * sizeof(uint64_t)));
        }
        const int col0 = n0 + cb * 32;
        if (row >= M || col0 >= N) continue;
        bf16* dst = out + (long long)row * ldo + col0;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          if (col0 + 8 * v >= N) break;
          uint4 pk;
          uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float x0 = __uint_as_float(r[8 * v + 2 * e]);
            float x1 = __uint_as_float(r[8 * v + 2 * e + 1]);
            if constexpr (FP8) {
              x0 = (x0 * scale_a) * scale_b;  // (acc * sx) * sw, fp8_emul.py:87
              x1 = (x1 * scale_a) * scale_b;
            } else {
              if (bias != nullptr) {
                x0 += __bfloat162float(bias[col0 + 8 * v + 2 * e]);
                x1 += __bfloat162float(bias[col0 + 8 * v + 2 * e + 1]);
              }
            }
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
            pw[e] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          st_stream16(dst + 8 * v, pk);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  // the pair's MMAs, copies and remote arrivals are over before either CTA
  // releases tensor memory or exits
  cluster_arrive();
  cluster_wait();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(Cfg2::TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

static int make_map(CUtensorMap* m, const void* base, bool fp8, uint64_t inner, uint64_t outer,
                    uint64_t ld_elems, uint32_t box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(HYENA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const int elem = fp8 ? 1 : 2;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * elem};
  cuuint32_t box[2] = {uint32_t(BKB / elem), box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      fn(m, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HYENA_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  return HYENA_OK;
}

// Upper bound on the CTAs of a persistent GEMM (0 = one per SM): leaves SMs
// free for kernels that must run alongside, such as collectives on another
// stream.  Set through hyena_set_gemm_max_ctas.
static std::atomic<int> g_max_ctas{0};

template <bool FP8, int BN>
static int launch_bn(const CUtensorMap& ta, const void* B, int64_t ldb, void* out, int64_t ldo,
                     int M, int N, int K, const float* sa, const float* sb, const void* bias,
                     cudaStream_t st) {
  CUtensorMap tb;
  int rc = make_map(&tb, B, FP8, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BN);
  if (rc) return rc;
  const size_t smem = sizeof(Smem<BN>) + 1024;
  if (!smem_attr<gemm_kernel<FP8, BN>>((int)smem)) return fail(HYENA_ERR_CUDA, "cudaFuncSetAttribute(gemm) failed");
  const long long tiles = (long long)((N + BN - 1) / BN) * ((M + BM - 1) / BM);
  long long cap = num_sms();
  const int lim = g_max_ctas.load(std::memory_order_relaxed);
  if (lim > 0 && lim < cap) cap = lim;
  dim3 grid((unsigned)(tiles < cap ? tiles : cap));
  launch_kernel(gemm_kernel<FP8, BN>, dim3(grid), dim3(THREADS), smem, st, 0u, ta, tb, static_cast<bf16*>(out), ldo, M, N,
                                                    K, sa, sb, static_cast<const bf16*>(bias));
  return check_launch(FP8 ? "gemm_kernel<e4m3>" : "gemm_kernel<bf16>");
}

template <bool FP8, int BN>
static size_t cluster_smem() {
  return sizeof(SmemSK<BN>) + 1024;
}

template <bool FP8, int BN>
static bool cluster_attr() {
  return smem_attr<gemm_cluster_kernel<FP8, BN>>((int)cluster_smem<FP8, BN>());
}

// How many clusters of `splits` CTAs can be resident at once (0 if unknown).
template <bool FP8, int BN>
static int resident_clusters(int splits) {
  static int cache[9] = {-1, -1, -1, -1, -1, -1, -1, -1, -1};
  if (splits < 1 || splits > 8) return 0;
  if (cache[splits] < 0) {
    int n = 0;
    if (cluster_attr<FP8, BN>()) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)splits, 1, 1);
      cfg.blockDim = dim3(THREADS, 1, 1);
      cfg.dynamicSmemBytes = cluster_smem<FP8, BN>();
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = (unsigned)splits;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, gemm_cluster_kernel<FP8, BN>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    cache[splits] = n;
  }
  return cache[splits];
}

template <bool FP8, int BN>
static int launch_cluster(const CUtensorMap& ta, const void* B, int64_t ldb, void* out,
                          int64_t ldo, int M, int N, int K, const float* sa, const float* sb,
                          const void* bias, int splits, cudaStream_t st) {
  CUtensorMap tb;
  int rc = make_map(&tb, B, FP8, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BN);
  if (rc) return rc;
  if (!cluster_attr<FP8, BN>()) return fail(HYENA_ERR_CUDA, "cudaFuncSetAttribute(gemm_cluster) failed");
  const int tiles = ((N + BN - 1) / BN) * ((M + BM - 1) / BM);
  launch_kernel(gemm_cluster_kernel<FP8, BN>, dim3((unsigned)splits, (unsigned)tiles, 1),
                dim3(THREADS), cluster_smem<FP8, BN>(), st, (unsigned)splits, ta, tb,
                static_cast<bf16*>(out), ldo, M, N, K, sa, sb, static_cast<const bf16*>(bias));
  return check_launch(FP8 ? "gemm_cluster_kernel<e4m3>" : "gemm_cluster_kernel<bf16>");
}

template <bool FP8>
static int launch_pair(const CUtensorMap& ta, const void* B, int64_t ldb, void* out, int64_t ldo,
                       int M, int N, int K, const float* sa, const float* sb, const void* bias,
                       cudaStream_t st) {
  CUtensorMap tb;
  int rc = make_map(&tb, B, FP8, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BN2 / 2);
  if (rc) return rc;
  const size_t smem = sizeof(Smem2) + 1024;
  if (!smem_attr<gemm_pair_kernel<FP8>>((int)smem))
    return fail(HYENA_ERR_CUDA, "cudaFuncSetAttribute(gemm_pair) failed");
  const long long tiles = (long long)((N + BN2 - 1) / BN2) * ((M + 2 * BM - 1) / (2 * BM));
  // the pairs that can be resident at once (SM pairs are formed inside a GPC,
  // so this can be below half the SMs): a pair launched beyond them would
  // start its statically assigned tiles only after another pair finished
  static int resident_pairs[2] = {-1, -1};
  int& rp = resident_pairs[FP8 ? 1 : 0];
  if (rp < 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<FP8>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    rp = n;
  }
  long long cap = rp;
  const int lim = g_max_ctas.load(std::memory_order_relaxed);
  if (lim > 0 && lim / 2 < cap) cap = lim / 2 > 0 ? lim / 2 : 1;
  dim3 grid((unsigned)(2 * (tiles < cap ? tiles : cap)));
  // Launched without programmatic stream serialisation: its CTAs start only
  // once the previous kernel in the stream has completed.  (Its own dependents
  // may still launch early.)  Launched as a programmatic dependent, so that its
  // pairs became resident beside the previous kernel's still-running CTAs, the
  // prefill step stalled for good within a few steps, with no bounded wait of
  // this kernel expiring; launched this way it ran clean.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, gemm_pair_kernel<FP8>, ta, tb, static_cast<bf16*>(out), ldo, M, N, K,
                     sa, sb, static_cast<const bf16*>(bias));
  return check_launch(FP8 ? "gemm_pair_kernel<e4m3>" : "gemm_pair_kernel<bf16>");
}

struct Plan {
  int bn, splits;  // splits > 0: cluster kernel with that many K slices per tile
  bool pair = false;  // 256 x 256 tiles on SM pairs (gemm_pair_kernel)
};

// Rows from which the SM-pair kernel takes over: enough 256-row tiles that
// every pair has several and the last wave is short.
constexpr int PAIR_MIN_M = 4096;

template <bool FP8>
static int resident(int bn, int splits) {
  switch (bn) {
    case 256: return resident_clusters<FP8, 256>(splits);
    case 192: return resident_clusters<FP8, 192>(splits);
    case 128: return resident_clusters<FP8, 128>(splits);
    default: return resident_clusters<FP8, 64>(splits);
  }
}

// Large M: the persistent kernel (splits = 0) with the N-tile width that gives
// every SM a tile and the shortest last wave: cost = waves x (BN + 32), the 32
// standing for a tile's fixed epilogue share; 256 unless another width is at
// least 10% cheaper (M = 512 x N = 12288: 192-wide tiles, 256 tiles in 2 waves
// instead of 192 tiles whose second wave is nearly as long as the first).  Small M (decode batches): the cluster kernel with the
// (BN, splits) that, in one resident wave of at most one CTA per SM, puts the
// fewest operand bytes through any one SM ((BM + BN) x its K slice; ties: fewer
// splits), each K slice at least two stages long.
template <bool FP8>
static Plan plan(int M, int N, int K) {
  const long long mt = (M + BM - 1) / BM;
  const int sms = num_sms();
  if (M >= PAIR_MIN_M && N >= BN2) return {BN2, 0, true};
  {
    int pick = 0;
    long long pick_cost = 0, cost256 = -1;
    for (int bn : {256, 192, 128}) {
      const long long tiles = mt * ((N + bn - 1) / bn);
      if (tiles < sms) continue;
      const long long cost = ((tiles + sms - 1) / sms) * (bn + 32);
      if (bn == 256) cost256 = cost;
      if (pick == 0 || cost < pick_cost) {
        pick = bn;
        pick_cost = cost;
      }
    }
    if (pick != 0 && cost256 >= 0 && pick != 256 && 10 * pick_cost > 9 * cost256) pick = 256;
    if (pick != 0) return {pick, 0};
  }
  const int kblocks = K / (BKB / (FP8 ? 1 : 2));
  Plan best = {0, 0};
  long long best_cost = 0;
  for (int bn : {256, 192, 128, 64}) {
    const long long tiles = mt * ((N + bn - 1) / bn);
    for (int sp = 1; sp <= 8; ++sp) {
      if (tiles * sp > sms || sp > (bn >= 256 ? max_cluster_splits<256>() : max_cluster_splits<128>()))
        break;
      if (sp > 1 && kblocks / sp < 2) break;
      if (resident<FP8>(bn, sp) < tiles) continue;
      const long long cost = (long long)(BM + bn) * ((kblocks + sp - 1) / sp);
      if (best.splits == 0 || cost < best_cost || (cost == best_cost && sp < best.splits)) {
        best = {bn, sp};
        best_cost = cost;
      }
    }
  }
  if (best.splits > 0) return best;
  return {mt * ((N + 63) / 64) >= sms ? 64 : 32, 0};
}

template <bool FP8>
static int launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* out, int64_t ldo,
                  int M, int N, int K, const float* sa, const float* sb, const void* bias,
                  cudaStream_t st) {
  if (M <= 0 || N <= 0) return HYENA_OK;
  const int KE = BKB / (FP8 ? 1 : 2);
  HB_REQUIRE(K > 0 && K % KE == 0, FP8 ? "e4m3 GEMM needs K % 128 == 0" : "bf16 GEMM needs K % 64 == 0");
  HB_REQUIRE(N % 8 == 0 && ldo % 8 == 0, "GEMM needs N % 8 == 0 and ldo % 8 == 0");
  HB_REQUIRE(aligned16(A) && aligned16(B) && aligned16(out), "GEMM operands must be 16-byte aligned");
  HB_REQUIRE((lda * (FP8 ? 1 : 2)) % 16 == 0 && (ldb * (FP8 ? 1 : 2)) % 16 == 0,
             "GEMM row strides must be multiples of 16 bytes");
  HB_REQUIRE(lda >= K && ldb >= K && ldo >= N, "GEMM leading dimensions too small");
  CUtensorMap ta;
  int rc = make_map(&ta, A, FP8, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BM);
  if (rc) return rc;
  const Plan pl = plan<FP8>(M, N, K);
  if (pl.pair) return launch_pair<FP8>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, st);
  if (pl.splits > 0) {
    switch (pl.bn) {
      case 256:
        return launch_cluster<FP8, 256>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, pl.splits, st);
      case 192:
        return launch_cluster<FP8, 192>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, pl.splits, st);
      case 128:
        return launch_cluster<FP8, 128>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, pl.splits, st);
      default:
        return launch_cluster<FP8, 64>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, pl.splits, st);
    }
  }
  switch (pl.bn) {
    case 256: return launch_bn<FP8, 256>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, st);
    case 192: return launch_bn<FP8, 192>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, st);
    case 128: return launch_bn<FP8, 128>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, st);
    case 64: return launch_bn<FP8, 64>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, st);
    default: return launch_bn<FP8, 32>(ta, B, ldb, out, ldo, M, N, K, sa, sb, bias, st);
  }
}

}  // namespace gemm

// `ws` / `ws_bytes` are accepted for ABI stability and not used: small-M
// calls reduce their K slices inside a cluster.
int gemm_e4m3_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                     int64_t ldo, int M, int N, int K, const float* sa, const float* sb,
                     void* ws, size_t ws_bytes, cudaStream_t st) {
  (void)ws;
  (void)ws_bytes;
  return gemm::launch<true>(A, lda, B, ldb, out, ldo, M, N, K, sa, sb, nullptr, st);
}

int gemm_bf16_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                     int64_t ldo, int M, int N, int K, const void* bias, void* ws,
                     size_t ws_bytes, cudaStream_t st) {
  (void)ws;
  (void)ws_bytes;
  return gemm::launch<false>(A, lda, B, ldb, out, ldo, M, N, K, nullptr, nullptr, bias, st);
}

void gemm_set_max_ctas(int n) { gemm::g_max_ctas.store(n > 0 ? n : 0, std::memory_order_relaxed); }

// Expired mbarrier waits counted on the current device since the last reset
// (a synchronous copy of the device counter; not for use inside a capture).
int gemm_wait_timeouts(int32_t* count, int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, gemm::g_wait_timeouts, sizeof(int));
  if (e != cudaSuccess)
    return fail(HYENA_ERR_CUDA, std::string("gemm wait counter read: ") + cudaGetErrorString(e));
  if (reset && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(gemm::g_wait_timeouts, &zero, sizeof(int));
    if (e != cudaSuccess)
      return fail(HYENA_ERR_CUDA, std::string("gemm wait counter reset: ") + cudaGetErrorString(e));
  }
  *count = v;
  return HYENA_OK;
}

size_t gemm_workspace_size(int M, int N, int K, bool fp8) {
  (void)M;
  (void)N;
  (void)K;
  (void)fp8;
  return 0;
}

}  // namespace hb
