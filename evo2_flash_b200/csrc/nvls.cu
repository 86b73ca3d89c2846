// In-switch all-reduce of the row-parallel out_proj partial sums over the
// ranks of one NVSwitch node (NVLink SHARP), for the channel-sharded mixer.
//
// Every rank's partial (T, H) bf16 output lives in a symmetric buffer that is
// also mapped as one NVLink multicast object.  Rank r owns the r-th slice of
// the buffer's 16-byte vectors: for each vector of its slice it issues one
// multimem.ld_reduce (the switch reads that vector from every rank's buffer,
// sums in fp32 and returns the bf16 result) and one multimem.st (the switch
// writes the result into every rank's buffer).  So each rank moves about one
// buffer's worth of bytes over NVLink in each direction, no SM does any
// arithmetic on the data, and the kernel needs only a few CTAs: it is made to
// run beside the compute kernels on a separate stream.  The sum is rounded to
// bf16 once (an NCCL ring rounds after every hop).
//
// Ordering: CTA b of every rank handshakes with CTA b of every other rank
// before reading (every partial is complete) and after writing (every result
// has landed), through flags in the ranks' signal pads: slot
// (phase, b, source rank) of a pad holds the epoch of the last call in which
// the source passed that point.  Epochs only grow, so a rank that is one call
// ahead never blocks one that is behind.  Every wait is bounded: on expiry the
// CTA sets HYENA_FLAG_COLLECTIVE in the error word and returns.
#include "common.cuh"

namespace hb {

constexpr int NV_THREADS = 512;
constexpr int NV_UNROLL = 4;              // 16-byte vectors in flight per thread
constexpr long long NV_SPIN_LIMIT = 1LL << 24;  // ~1 s with the 64 ns back-off

__device__ __forceinline__ void nv_st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t nv_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Tells every rank that this CTA passed point `phase` of call `epoch` and waits
// until every rank's CTA b did the same.  Every thread's earlier accesses
// (through either address alias) are ordered before the note by its own fences
// and the CTA barrier, and no thread's later access starts before the waits
// ended.  False when a wait expired.
__device__ bool nv_handshake(uint32_t* const* pads, int rank, int world, int phase,
                             uint32_t epoch) {
  asm volatile("fence.proxy.alias;" ::: "memory");
  __threadfence_system();
  __syncthreads();
  bool ok = true;
  const int b = blockIdx.x, nb = gridDim.x;
  if (threadIdx.x < world) {
    const int t = threadIdx.x;
    nv_st_release(pads[t] + ((size_t)(phase * nb + b) * world + rank), epoch);
    const uint32_t* mine = pads[rank] + ((size_t)(phase * nb + b) * world + t);
    long long it = 0;
    while ((int32_t)(nv_ld_acquire(mine) - epoch) < 0) {
      if (++it > NV_SPIN_LIMIT) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  ok = __syncthreads_and(ok) != 0;
  asm volatile("fence.proxy.alias;" ::: "memory");
  return ok;
}

__global__ void __launch_bounds__(NV_THREADS)
nvls_allreduce_kernel(uint4* mc, long long nvec, uint32_t* const* pads, int rank, int world,
                      uint32_t epoch, int32_t* err) {
  pdl_entry();
  if (!nv_handshake(pads, rank, world, 0, epoch)) {
    if (threadIdx.x == 0) flag_error(err, HYENA_FLAG_COLLECTIVE);
    return;
  }
  const long long per_rank = (nvec + world - 1) / world;
  const long long s0 = (long long)rank * per_rank;
  const long long s1 = min(nvec, s0 + per_rank);
  const long long stride = (long long)gridDim.x * NV_THREADS;
  for (long long i0 = s0 + (long long)blockIdx.x * NV_THREADS + threadIdx.x; i0 < s1;
       i0 += stride * NV_UNROLL) {
    uint4 v[NV_UNROLL];
#pragma unroll
    for (int u = 0; u < NV_UNROLL; ++u) {
      const long long i = i0 + u * stride;
      if (i < s1)
        asm volatile(
            "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
            : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
            : "l"(mc + i)
            : "memory");
    }
#pragma unroll
    for (int u = 0; u < NV_UNROLL; ++u) {
      const long long i = i0 + u * stride;
      if (i < s1)
        asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc + i),
                     "r"(v[u].x), "r"(v[u].y), "r"(v[u].z), "r"(v[u].w)
                     : "memory");
    }
  }
  if (!nv_handshake(pads, rank, world, 1, epoch) && threadIdx.x == 0)
    flag_error(err, HYENA_FLAG_COLLECTIVE);
}

}  // namespace hb

extern "C" int hyena_nvls_allreduce_bf16(void* multicast, int64_t n_elems, void* const* signal_pads,
                                          int64_t signal_pad_bytes, int32_t rank, int32_t world,
                                          uint32_t epoch, int32_t num_ctas, int32_t* error_flags,
                                          void* stream) {
  using namespace hb;
  HB_REQUIRE(multicast != nullptr && signal_pads != nullptr, "null multicast or signal pads");
  HB_REQUIRE(aligned16(multicast) && n_elems % 8 == 0, "buffer must be 16-byte aligned, n % 8 == 0");
  HB_REQUIRE(world >= 1 && world <= 64 && rank >= 0 && rank < world, "bad rank / world");
  HB_REQUIRE(num_ctas >= 1 && num_ctas <= 128, "num_ctas must be in [1, 128]");
  HB_REQUIRE(epoch != 0, "epoch must be nonzero (pads start at zero)");
  HB_REQUIRE(2LL * num_ctas * world * (long long)sizeof(uint32_t) <= signal_pad_bytes,
             "signal pads too small for 2 x num_ctas x world flags");
  if (n_elems == 0) return HYENA_OK;
  // the launch is not chained to the stream's previous kernel: this runs on a
  // collective stream whose predecessor is another rank-wide handshake
  nvls_allreduce_kernel<<<num_ctas, NV_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(multicast), (long long)(n_elems / 8),
      reinterpret_cast<uint32_t* const*>(signal_pads), rank, world, epoch, error_flags);
  return check_launch("nvls_allreduce_kernel");
}
