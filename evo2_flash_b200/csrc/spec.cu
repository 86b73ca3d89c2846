// Speculative-decoding bookkeeping on the position stamps (one fp32 per state
// block, the last column of S2's first channel: mixers.py:952-957): accepted
// counts, verifier-slot and prefill stamps, and the prefix-caching repair of
// resumed prefill rows, each a small kernel in place of the reference's chain
// of torch ops (mixers.py:962-984, 1001-1074).  Stamps are exact integers in
// fp32 (< 2^24).
#include <algorithm>

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

// Prefix-caching repair of resumed prefill rows (the defect the reference
// guards against at mixers.py:1001-1037): a prefill row that continues from
// `computed` tokens must start from a block stamped `computed`.  When its
// destination block is not, but the source block of its last computed token
// is, the whole state of the source block (all slices) is copied over the
// destination.  Phase 1 decides every row from the stamps as they are before
// any copy; phase 2 copies.  take[j] = source block, or -1 (no copy).
__global__ void __launch_bounds__(128)
state_repair_decide_kernel(int num_rows, const int32_t* __restrict__ dst, int64_t dst_stride,
                           const int32_t* __restrict__ src, const int32_t* __restrict__ computed,
                           const uint8_t* __restrict__ has_init, const float* __restrict__ stamps,
                           int64_t stamp_stride, int num_blocks, int32_t* __restrict__ take,
                           int32_t* error_flags) {
  pdl_entry();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= num_rows) return;
  const long long d = __ldg(dst + (long long)j * dst_stride);
  const long long s = __ldg(src + j);
  int32_t pick = -1;
  if (has_init[j] != 0 && d != 0 && s != 0) {
    if (d < 0 || d >= num_blocks || s < 0 || s >= num_blocks) {
      flag_error(error_flags, HYENA_FLAG_BLOCK_RANGE);
    } else {
      const float want = (float)__ldg(computed + j);
      const bool dst_stale = __ldg(stamps + d * stamp_stride) != want;
      const bool src_good = __ldg(stamps + s * stamp_stride) == want;
      if (dst_stale && src_good) pick = (int32_t)s;
    }
  }
  take[j] = pick;
}

// Phase 2: blockIdx.x = row, blockIdx.y = slice, blockIdx.z = part of the
// slice; 16-byte copies.
__global__ void __launch_bounds__(256)
state_repair_copy_kernel(int num_rows, const int32_t* __restrict__ dst, int64_t dst_stride,
                         const int32_t* __restrict__ take, hyena_state_block s0,
                         hyena_state_block s1, hyena_state_block s2) {
  pdl_entry();
  const int j = blockIdx.x;
  const long long from = __ldg(take + j);
  if (from < 0) return;
  const long long to = __ldg(dst + (long long)j * dst_stride);
  const hyena_state_block& sl = blockIdx.y == 0 ? s0 : blockIdx.y == 1 ? s1 : s2;
  if (sl.data == nullptr) return;
  const long long n16 = sl.block_bytes / 16;
  const uint4* a = reinterpret_cast<const uint4*>(static_cast<const char*>(sl.data) +
                                                  from * sl.block_stride_bytes);
  uint4* b = reinterpret_cast<uint4*>(static_cast<char*>(sl.data) + to * sl.block_stride_bytes);
  for (long long i = (long long)blockIdx.z * blockDim.x + threadIdx.x; i < n16;
       i += (long long)gridDim.z * blockDim.x)
    b[i] = a[i];
}

// stamp(blocks[j]) = seq_lens[j] for the prefill rows of a step (the prefill
// half of the reference's _record_stamps, mixers.py:1070-1074).
__global__ void __launch_bounds__(128)
spec_record_prefill_kernel(const int32_t* __restrict__ blocks, int64_t block_stride, int n,
                           const int32_t* __restrict__ seq_lens, float* __restrict__ stamps,
                           int64_t stamp_stride, int num_blocks, int32_t* error_flags) {
  pdl_entry();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const long long b = __ldg(blocks + (long long)j * block_stride);
  if (b < 0 || b >= num_blocks) {
    flag_error(error_flags, HYENA_FLAG_BLOCK_RANGE);
    return;
  }
  stamps[b * stamp_stride] = (float)__ldg(seq_lens + j);
}

int state_repair_launch(int num_rows, const int32_t* dst, int64_t dst_stride, const int32_t* src,
                        const int32_t* computed, const uint8_t* has_init, const float* stamps,
                        int64_t stamp_stride, int num_blocks, const hyena_state_block* slices,
                        int num_slices, int32_t* take, int32_t* error_flags, cudaStream_t st) {
  if (num_rows <= 0) return HYENA_OK;
  HB_REQUIRE(dst && src && computed && has_init && stamps && take && slices,
             "state_repair: null pointer");
  HB_REQUIRE(num_slices >= 1 && num_slices <= 3, "state_repair: 1 to 3 state slices");
  HB_REQUIRE(num_blocks > 0, "state_repair: no blocks");
  hyena_state_block sl[3] = {};
  long long most = 0;
  for (int i = 0; i < num_slices; ++i) {
    sl[i] = slices[i];
    if (sl[i].data == nullptr) continue;
    HB_REQUIRE(aligned16(sl[i].data) && sl[i].block_stride_bytes % 16 == 0 &&
                   sl[i].block_bytes % 16 == 0 && sl[i].block_bytes >= 0 &&
                   sl[i].block_bytes <= sl[i].block_stride_bytes,
               "state_repair: slices need 16-byte aligned blocks of whole 16-byte words");
    if (sl[i].block_bytes > most) most = sl[i].block_bytes;
  }
  launch_kernel(state_repair_decide_kernel, dim3((num_rows + 127) / 128), dim3(128), 0, st, 0u,
                num_rows, dst, dst_stride, src, computed, has_init, stamps, stamp_stride,
                num_blocks, take, error_flags);
  int rc = check_launch("state_repair_decide_kernel");
  if (rc) return rc;
  const long long words = most / 16;
  const int parts = (int)std::min<long long>(64, std::max<long long>(1, (words + 4095) / 4096));
  launch_kernel(state_repair_copy_kernel, dim3(num_rows, 3, parts), dim3(256), 0, st, 0u,
                num_rows, dst, dst_stride, (const int32_t*)take, sl[0], sl[1], sl[2]);
  return check_launch("state_repair_copy_kernel");
}

int spec_record_prefill_launch(const int32_t* blocks, int64_t block_stride, int n,
                               const int32_t* seq_lens, float* stamps, int64_t stamp_stride,
                               int num_blocks, int32_t* error_flags, cudaStream_t st) {
  if (n <= 0) return HYENA_OK;
  HB_REQUIRE(blocks && seq_lens && stamps, "spec_record_prefill: null pointer");
  launch_kernel(spec_record_prefill_kernel, dim3((n + 127) / 128), dim3(128), 0, st, 0u, blocks,
                block_stride, n, seq_lens, stamps, stamp_stride, num_blocks, error_flags);
  return check_launch("spec_record_prefill_kernel");
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
