// Speculative-decoding bookkeeping on the position stamps (one fp32 per state
// block, the last column of S2's first channel: mixers.py:952-957), as two
// one-thread-per-request kernels in place of the reference's chain of small
// torch ops (mixers.py:962-984, 1040-1062).  Stamps are exact integers in fp32
// (< 2^24).
#include "common.cuh"

namespace hb {

__global__ void __launch_bounds__(128)
spec_accepted_kernel(const int32_t* __restrict__ slots, int64_t slot_stride, int num_reqs,
                     const int32_t* __restrict__ computed, const float* __restrict__ stamps,
                     int64_t stamp_stride, int num_blocks, int num_spec,
                     int32_t* __restrict__ accepted, int32_t* error_flags) {
  pdl_entry();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= num_reqs) return;
  const long long first = __ldg(slots + (long long)r * slot_stride);
  long long offset = 0;
  if (first >= 0 && first < num_blocks) {
    offset = (long long)__ldg(computed + r) - (long long)__ldg(stamps + first * stamp_stride);
    if (first != 0 && (offset < 0 || offset > num_spec)) flag_error(error_flags, HYENA_FLAG_STAMP);
  } else {
    flag_error(error_flags, HYENA_FLAG_BLOCK_RANGE);
  }
  accepted[r] = (int32_t)(offset < 0 ? 0 : offset > num_spec ? num_spec : offset) + 1;
}

__global__ void __launch_bounds__(128)
spec_record_kernel(const int32_t* __restrict__ out_slots, int64_t s0, int64_t s1, int num_reqs,
                   int q, const int32_t* __restrict__ starts, const int32_t* __restrict__ computed,
                   float* __restrict__ stamps, int64_t stamp_stride, int num_blocks,
                   int32_t* error_flags) {
  pdl_entry();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= num_reqs) return;
  const int len = __ldg(starts + r + 1) - __ldg(starts + r);
  const long long c = __ldg(computed + r);
  for (int p = 0; p < q && p < len; ++p) {
    const long long b = __ldg(out_slots + (long long)r * s0 + (long long)p * s1);
    if (b == 0) continue;  // the null block's stamp is never consulted
    if (b < 0 || b >= num_blocks) {
      flag_error(error_flags, HYENA_FLAG_BLOCK_RANGE);
      continue;
    }
    stamps[b * stamp_stride] = (float)(c + p + 1);
  }
}

int spec_accepted_launch(const int32_t* slots, int64_t slot_stride, int num_reqs,
                         const int32_t* computed, const float* stamps, int64_t stamp_stride,
                         int num_blocks, int num_spec, int32_t* accepted, int32_t* error_flags,
                         cudaStream_t st) {
  if (num_reqs <= 0) return HYENA_OK;
  HB_REQUIRE(slots && computed && stamps && accepted, "spec_accepted: null pointer");
  HB_REQUIRE(num_spec >= 0 && num_blocks > 0, "spec_accepted: bad num_spec / num_blocks");
  launch_kernel(spec_accepted_kernel, dim3((num_reqs + 127) / 128), dim3(128), 0, st, 0u, slots,
                slot_stride, num_reqs, computed, stamps, stamp_stride, num_blocks, num_spec,
                accepted, error_flags);
  return check_launch("spec_accepted_kernel");
}

int spec_record_launch(const int32_t* out_slots, int64_t s0, int64_t s1, int num_reqs, int q,
                       const int32_t* starts, const int32_t* computed, float* stamps,
                       int64_t stamp_stride, int num_blocks, int32_t* error_flags,
                       cudaStream_t st) {
  if (num_reqs <= 0 || q <= 0) return HYENA_OK;
  HB_REQUIRE(out_slots && starts && computed && stamps, "spec_record: null pointer");
  launch_kernel(spec_record_kernel, dim3((num_reqs + 127) / 128), dim3(128), 0, st, 0u, out_slots,
                s0, s1, num_reqs, q, starts, computed, stamps, stamp_stride, num_blocks,
                error_flags);
  return check_launch("spec_record_kernel");
}

}  // namespace hb
