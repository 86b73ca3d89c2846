// C ABI entry points: argument validation, dispatch, thread-local error text.
#include <atomic>
#include <cmath>
#include <cstdio>

#include "common.cuh"

namespace hb {

static thread_local std::string g_last_error;
static std::atomic<bool> g_launch_chaining{true};

bool launch_chaining() { return g_launch_chaining.load(std::memory_order_relaxed); }

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return HYENA_OK;
  return fail(HYENA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int fir_prefill_launch(const hyena_layer_params& P, const hyena_prefill_args& A, cudaStream_t st);
int hcl_prefill_launch(const hyena_layer_params& P, const hyena_prefill_args& A, void* ws,
                       size_t ws_bytes, cudaStream_t st);
size_t hcl_workspace_size(int H, int T, int nseg);
int decode_launch(const hyena_layer_params& P, const hyena_decode_args& A, cudaStream_t st);
int quant_e4m3_launch(const void* x, int64_t ldx, void* q, int64_t ldq, int M, int K,
                      const float* scale, cudaStream_t st);
int gemm_e4m3_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                     int64_t ldo, int M, int N, int K, const float* sa, const float* sb,
                     void* ws, size_t ws_bytes, cudaStream_t st);
int gemm_bf16_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                     int64_t ldo, int M, int N, int K, const void* bias, void* ws,
                     size_t ws_bytes, cudaStream_t st);
size_t gemm_workspace_size(int M, int N, int K, bool fp8);
int gemm_fp8_emulated_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                             int64_t ldo, int N, int M, int K, const float* sa, const float* sb,
                             cudaStream_t st);
void gemm_set_max_ctas(int n);
int gemm_wait_timeouts(int32_t* count, int reset);
int spec_accepted_launch(const int32_t* slots, int64_t slot_stride, int num_reqs,
                         const int32_t* computed, const float* stamps, int64_t stamp_stride,
                         int num_blocks, int num_spec, int32_t* accepted, int32_t* error_flags,
                         cudaStream_t st);
int spec_record_launch(const int32_t* out_slots, int64_t s0, int64_t s1, int num_reqs, int q,
                       const int32_t* starts, const int32_t* computed, float* stamps,
                       int64_t stamp_stride, int num_blocks, int32_t* error_flags,
                       cudaStream_t st);

int state_repair_launch(int num_rows, const int32_t* dst, int64_t dst_stride, const int32_t* src,
                        const int32_t* computed, const uint8_t* has_init, const float* stamps,
                        int64_t stamp_stride, int num_blocks, const hyena_state_block* slices,
                        int num_slices, int32_t* take, int32_t* error_flags, cudaStream_t st);
int spec_record_prefill_launch(const int32_t* blocks, int64_t block_stride, int n,
                               const int32_t* seq_lens, float* stamps, int64_t stamp_stride,
                               int num_blocks, int32_t* error_flags, cudaStream_t st);

static int check_params(const hyena_layer_params* p) {
  HB_REQUIRE(p != nullptr, "null layer params");
  HB_REQUIRE(p->H > 0 && p->H % 64 == 0, "H must be a positive multiple of 64");
  HB_REQUIRE(p->short_w != nullptr, "short_w is null");
  if (p->kind == HYENA_KIND_FIR) {
    HB_REQUIRE(p->inner_w != nullptr, "FIR inner_w is null");
    HB_REQUIRE(p->K == 7 || p->K == 128, "FIR K must be 7 or 128");
  } else if (p->kind == HYENA_KIND_IIR) {
    HB_REQUIRE(p->log_poles != nullptr && p->residues != nullptr, "IIR poles/residues are null");
    HB_REQUIRE(p->K == 16, "IIR modal order must be 16");
  } else {
    return fail(HYENA_ERR_INVALID, "unknown mixer kind");
  }
  return HYENA_OK;
}

static int check_view(const hyena_state_view& v, const char* name, int min_cols) {
  if (v.data == nullptr) return fail(HYENA_ERR_INVALID, std::string(name) + ": null data");
  if (v.cols < min_cols)
    return fail(HYENA_ERR_INVALID, std::string(name) + ": too few window columns");
  if (v.num_blocks <= 0) return fail(HYENA_ERR_INVALID, std::string(name) + ": no blocks");
  return HYENA_OK;
}

}  // namespace hb

using namespace hb;

extern "C" {

int hyena_abi_version(void) { return HYENA_ABI_VERSION; }

void hyena_set_gemm_max_ctas(int32_t n) { hb::gemm_set_max_ctas(n); }

int hyena_spec_accepted(const int32_t* slots, int64_t slot_stride, int32_t num_reqs,
                        const int32_t* computed, const float* stamps, int64_t stamp_stride,
                        int32_t num_blocks, int32_t num_spec, int32_t* accepted,
                        int32_t* error_flags, void* stream) {
  return hb::spec_accepted_launch(slots, slot_stride, num_reqs, computed, stamps, stamp_stride,
                                  num_blocks, num_spec, accepted, error_flags,
                                  static_cast<cudaStream_t>(stream));
}

int hyena_spec_record(const int32_t* out_slots, int64_t s0, int64_t s1, int32_t num_reqs,
                      int32_t q, const int32_t* starts, const int32_t* computed, float* stamps,
                      int64_t stamp_stride, int32_t num_blocks, int32_t* error_flags,
                      void* stream) {
  return hb::spec_record_launch(out_slots, s0, s1, num_reqs, q, starts, computed, stamps,
                                stamp_stride, num_blocks, error_flags,
                                static_cast<cudaStream_t>(stream));
}

int hyena_spec_record_prefill(const int32_t* blocks, int64_t block_stride, int32_t n,
                              const int32_t* seq_lens, float* stamps, int64_t stamp_stride,
                              int32_t num_blocks, int32_t* error_flags, void* stream) {
  return hb::spec_record_prefill_launch(blocks, block_stride, n, seq_lens, stamps, stamp_stride,
                                        num_blocks, error_flags,
                                        static_cast<cudaStream_t>(stream));
}

int hyena_state_repair(int32_t num_rows, const int32_t* dst_blocks, int64_t dst_stride,
                       const int32_t* src_blocks, const int32_t* computed,
                       const uint8_t* has_init, const float* stamps, int64_t stamp_stride,
                       int32_t num_blocks, const hyena_state_block* slices, int32_t num_slices,
                       int32_t* take, int32_t* error_flags, void* stream) {
  return hb::state_repair_launch(num_rows, dst_blocks, dst_stride, src_blocks, computed, has_init,
                                 stamps, stamp_stride, num_blocks, slices, num_slices, take,
                                 error_flags, static_cast<cudaStream_t>(stream));
}

void hyena_set_launch_chaining(int32_t enable) {
  hb::g_launch_chaining.store(enable != 0, std::memory_order_relaxed);
}

const char* hyena_last_error(void) { return g_last_error.c_str(); }

size_t hyena_prefill_workspace_size(const hyena_layer_params* p, int32_t T, int32_t nseg) {
  if (p == nullptr || p->kind != HYENA_KIND_IIR) return 0;
  return hcl_workspace_size(p->H, T < 0 ? 0 : T, nseg < 0 ? 0 : nseg);
}

int hyena_prefill(const hyena_layer_params* p, const hyena_prefill_args* a, void* ws,
                  size_t ws_bytes, void* stream) {
  int rc = check_params(p);
  if (rc) return rc;
  HB_REQUIRE(a != nullptr, "null prefill args");
  HB_REQUIRE(a->T >= 0 && a->num_segments >= 0, "negative sizes");
  if (a->T == 0 || a->num_segments == 0) return HYENA_OK;
  HB_REQUIRE(a->z && a->out && a->query_start_loc && a->state_indices, "null prefill pointer");
  HB_REQUIRE(aligned16(a->z) && a->ldz % 8 == 0, "z must be 16-byte aligned with ldz % 8 == 0");
  HB_REQUIRE(a->ldz >= 3LL * p->H && a->ldo >= p->H, "row strides too small");
  HB_REQUIRE((reinterpret_cast<uintptr_t>(a->out) & 3u) == 0 && a->ldo % 2 == 0,
             "out must be 4-byte aligned with an even row stride");
  if ((rc = check_view(a->conv_state, "conv_state", 2))) return rc;
  if (p->kind == HYENA_KIND_FIR) {
    if ((rc = check_view(a->inner_state, "inner_state", p->K - 1))) return rc;
  } else {
    if ((rc = check_view(a->inner_state, "inner_state", 16))) return rc;
  }
  HB_REQUIRE(a->conv_state.cols <= 8, "conv window wider than 8 columns");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p->kind == HYENA_KIND_FIR) return fir_prefill_launch(*p, *a, st);
  return hcl_prefill_launch(*p, *a, ws, ws_bytes, st);
}

int hyena_decode(const hyena_layer_params* p, const hyena_decode_args* a, void* stream) {
  int rc = check_params(p);
  if (rc) return rc;
  HB_REQUIRE(a != nullptr, "null decode args");
  if (a->num_reqs <= 0) return HYENA_OK;
  HB_REQUIRE(a->z && a->out && a->conv_in_block && a->conv_out_block && a->in_slots &&
                 a->out_slots,
             "null decode pointer");
  HB_REQUIRE(a->q >= 1 && a->q <= 8, "q must be in [1, 8]");
  HB_REQUIRE(a->ldz >= 3LL * p->H && a->ldo >= p->H, "row strides too small");
  if ((rc = check_view(a->conv_state, "conv_state", 2))) return rc;
  if ((rc = check_view(a->inner_state, "inner_state", p->kind == HYENA_KIND_FIR ? p->K - 1 : 16)))
    return rc;
  return decode_launch(*p, *a, static_cast<cudaStream_t>(stream));
}

int hyena_quant_e4m3(const void* x, int64_t ldx, void* q, int64_t ldq, int32_t M, int32_t K,
                     const float* input_scale, void* stream) {
  HB_REQUIRE(x && q && input_scale, "null quant pointer");
  return quant_e4m3_launch(x, ldx, q, ldq, M, K, input_scale, static_cast<cudaStream_t>(stream));
}

int hyena_gemm_e4m3(const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                    int64_t ldo, int32_t M, int32_t N, int32_t K, const float* scale_a,
                    const float* scale_b, void* workspace, size_t workspace_bytes,
                    void* stream) {
  HB_REQUIRE(A && B && out && scale_a && scale_b, "null gemm pointer");
  return gemm_e4m3_launch(A, lda, B, ldb, out, ldo, M, N, K, scale_a, scale_b, workspace,
                          workspace_bytes, static_cast<cudaStream_t>(stream));
}

int hyena_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                    int64_t ldo, int32_t M, int32_t N, int32_t K, const void* bias,
                    void* workspace, size_t workspace_bytes, void* stream) {
  HB_REQUIRE(A && B && out, "null gemm pointer");
  return gemm_bf16_launch(A, lda, B, ldb, out, ldo, M, N, K, bias, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream));
}

int hyena_rms_norm(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                   const void* weight, float eps, void* s_out, int64_t lds, void* y, int64_t ldy,
                   void* q, int64_t ldq, const float* input_scale, int32_t M, int32_t H,
                   void* stream) {
  HB_REQUIRE(M >= 0, "rms_norm: negative row count");
  hb::NormArgs A{static_cast<const bf16*>(x), ldx, static_cast<const bf16*>(residual), ldr,
                 static_cast<const bf16*>(weight), static_cast<bf16*>(s_out), lds,
                 static_cast<bf16*>(y), ldy, static_cast<uint8_t*>(q), ldq, input_scale, M, H,
                 // H ** -0.5 as a Python float, then the fp32 scalar torch multiplies by
                 static_cast<float>(std::pow(static_cast<double>(H), -0.5)), eps};
  return hb::rms_norm_launch(A, static_cast<cudaStream_t>(stream));
}

int hyena_gemm_fp8_emulated(const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                            int64_t ldo, int32_t N, int32_t M, int32_t K, const float* scale_a,
                            const float* scale_b, void* stream) {
  return hb::gemm_fp8_emulated_launch(A, lda, B, ldb, out, ldo, N, M, K, scale_a, scale_b,
                                      static_cast<cudaStream_t>(stream));
}

int hyena_gemm_wait_timeouts(int32_t* count, int32_t reset) {
  HB_REQUIRE(count != nullptr, "hyena_gemm_wait_timeouts: null count");
  return gemm_wait_timeouts(count, reset);
}

size_t hyena_gemm_workspace_size(int32_t M, int32_t N, int32_t K, int32_t fp8) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return gemm_workspace_size(M, N, K, fp8 != 0);
}

}  // extern "C"
