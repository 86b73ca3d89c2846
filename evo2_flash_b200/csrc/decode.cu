// Fused Hyena decode / speculative verify for sm_100a.
//
// One launch per Hyena layer per step handles every decode request:
//   K=3 short filter over the (x2, x1, v) triple from the cached S0 window at
//   column offset accepted-1, the shifted window written back (vLLM
//   causal_conv1d_update, incl. its speculative window convention);
//   u = bf16(x1*v);
//   inner operator from the snapshot in_slots[r, accepted-1]:
//     FIR (K=7 / 128): y_p = sum_k w[k] * win_p[k], one full (K-1)-window
//     snapshot written per verified position (mixers.py:578-628);
//     IIR (order 16): s = s*p + u without FMA, halving-tree readout, one modal
//     snapshot per position (mixers.py:631-663; triton_decode.py:81-96);
//   y = bf16(y) [+ bf16(D*u)], g = bf16(x2*y).
// Ordinary decode is the q = 1 case with in_slots == out_slots (in place,
// triton_decode.py:56-164).
//
// A thread owns one channel for one request, so every state element it writes
// is one it (and only it) has already read: the in-place shift of the FIR
// window streams the window once, writing each value one column lower, and all
// snapshot destinations are written at indices below the read position.
#include "common.cuh"

namespace hb {

constexpr int DEC_THREADS = 128;
constexpr int DEC_MAXQ = 8;
constexpr int DEC_MAXW0 = 8;

template <int N>
__device__ __forceinline__ float pick(const float (&v)[N], int i) {
  float r = 0.0f;
#pragma unroll
  for (int k = 0; k < N; ++k)
    if (k == i) r = v[k];
  return r;
}

__device__ __forceinline__ bool block_ok(long long b, const hyena_state_view& v) {
  return b >= 0 && b < v.num_blocks;
}

template <int KIND, int K>
__global__ void __launch_bounds__(DEC_THREADS)
decode_kernel(const hyena_layer_params P, const hyena_decode_args A) {
  const int r = blockIdx.x;
  const int h = blockIdx.y * DEC_THREADS + threadIdx.x;
  if (h >= P.H) return;

  int t0, n;
  if (A.token_start) {
    t0 = __ldg(A.token_start + r);
    n = __ldg(A.token_start + r + 1) - t0;
  } else {
    t0 = r;
    n = 1;
  }
  if (n <= 0) return;
  if (n > A.q || n > DEC_MAXQ) {
    if (threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_SEGMENT);
    n = min(A.q, DEC_MAXQ);
  }
  const int accepted = A.accepted ? max(1, __ldg(A.accepted + r)) : 1;
  const int off = accepted - 1;
  const long long cin = __ldg(A.conv_in_block + r);
  const long long cout = __ldg(A.conv_out_block + r);
  bf16* out = static_cast<bf16*>(A.out);
  const bf16* z = static_cast<const bf16*>(A.z);

  if ((A.zero_null_rows && cin == A.null_block) || !block_ok(cin, A.conv_state)) {
    if (!block_ok(cin, A.conv_state) && threadIdx.x == 0)
      flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
    for (int p = 0; p < n; ++p) out[(long long)(t0 + p) * A.ldo + h] = __float2bfloat16_rn(0.0f);
    return;
  }

  // ---- short filter on the triple, window shift
  const int W0 = A.conv_state.cols;
  bf16* s0 = static_cast<bf16*>(A.conv_state.data);
  const bf16* sw = static_cast<const bf16*>(P.short_w);
  const bool write_conv = block_ok(cout, A.conv_state) &&
                          !(A.skip_null_writes && cout == A.null_block);
  float xs[3][DEC_MAXQ];
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int col = 3 * h + q;
    const float w0 = ldbf(sw + col * 3), w1 = ldbf(sw + col * 3 + 1), w2 = ldbf(sw + col * 3 + 2);
    float win[DEC_MAXW0];
#pragma unroll
    for (int i = 0; i < DEC_MAXW0; ++i)
      win[i] = i < W0 ? ldbf(s0 + cin * A.conv_state.block_stride +
                             (long long)i * A.conv_state.col_stride +
                             (long long)col * A.conv_state.dim_stride)
                      : 0.0f;
    float c0 = off < W0 ? pick(win, off) : 0.0f;
    float c1 = off + 1 < W0 ? pick(win, off + 1) : 0.0f;
    float xz[DEC_MAXQ];
#pragma unroll
    for (int p = 0; p < DEC_MAXQ; ++p) {
      xz[p] = 0.0f;
      xs[q][p] = 0.0f;
      if (p < n) {
        xz[p] = ldbf(z + (long long)(t0 + p) * A.ldz + col);
        xs[q][p] = short_tap(c0, c1, xz[p], w0, w1, w2);
        c0 = c1;
        c1 = xz[p];
      }
    }
    if (write_conv) {
      const int val = W0 - n;  // columns kept from the old window
      for (int i = 0; i < W0; ++i) {
        float v;
        if (i < val) {
          const int src = off + 1 + i;
          v = src < W0 ? pick(win, src) : 0.0f;
        } else {
          v = pick(xz, i - val);
        }
        s0[cout * A.conv_state.block_stride + (long long)i * A.conv_state.col_stride +
           (long long)col * A.conv_state.dim_stride] = __float2bfloat16_rn(v);
      }
    }
  }
  float u[DEC_MAXQ];
#pragma unroll
  for (int p = 0; p < DEC_MAXQ; ++p) u[p] = bf16r(xs[1][p] * xs[2][p]);

  // ---- inner operator with snapshots
  const long long src = __ldg(A.in_slots + (long long)r * A.in_stride0 + (long long)off * A.in_stride1);
  long long dst[DEC_MAXQ];
  bool dok[DEC_MAXQ];
#pragma unroll
  for (int p = 0; p < DEC_MAXQ; ++p) {
    dst[p] = p < n ? __ldg(A.out_slots + (long long)r * A.out_stride0 + (long long)p * A.out_stride1) : 0;
    dok[p] = p < n && block_ok(dst[p], A.inner_state) &&
             !(A.skip_null_writes && dst[p] == A.null_block);
  }
  const bool src_ok = block_ok(src, A.inner_state);
  if (!src_ok && threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
  float y[DEC_MAXQ];
#pragma unroll
  for (int p = 0; p < DEC_MAXQ; ++p) y[p] = 0.0f;
  float* st = static_cast<float*>(A.inner_state.data);
  const long long cs = A.inner_state.col_stride;

  if constexpr (KIND == HYENA_KIND_FIR) {
    constexpr int HIST = K - 1;
    const bf16* w = static_cast<const bf16*>(P.inner_w) + (long long)h * P.inner_w_stride_h;
    const long long wk = P.inner_w_stride_k;
    const float* sp = st + src * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride;
    constexpr int CH = 8;
    for (int k0 = 0; k0 < HIST; k0 += CH) {
      float sv[CH];
#pragma unroll
      for (int t = 0; t < CH; ++t) sv[t] = (src_ok && k0 + t < HIST) ? sp[(long long)(k0 + t) * cs] : 0.0f;
#pragma unroll
      for (int t = 0; t < CH; ++t) {
        const int k = k0 + t;
        if (k < HIST) {
#pragma unroll
          for (int p = 0; p < DEC_MAXQ; ++p) {
            if (p < n && k >= p) y[p] = fmaf(ldbf(w + (long long)(k - p) * wk), sv[t], y[p]);
            if (p < n && dok[p] && k - p - 1 >= 0)
              st[dst[p] * A.inner_state.block_stride + (long long)(k - p - 1) * cs +
                 (long long)h * A.inner_state.dim_stride] = sv[t];
          }
        }
      }
    }
    // the verified tokens themselves: newest taps, and the tail of each snapshot
#pragma unroll
    for (int p = 0; p < DEC_MAXQ; ++p) {
      if (p < n) {
#pragma unroll
        for (int i = 0; i < DEC_MAXQ; ++i)
          if (i < p) y[p] = fmaf(ldbf(w + (long long)(HIST + i - p) * wk), u[i], y[p]);
        y[p] = fmaf(ldbf(w + (long long)HIST * wk), u[p], y[p]);
        if (dok[p]) {
#pragma unroll
          for (int m = 0; m < DEC_MAXQ; ++m)
            if (m <= p)
              st[dst[p] * A.inner_state.block_stride + (long long)(HIST - 1 - p + m) * cs +
                 (long long)h * A.inner_state.dim_stride] = u[m];
        }
      }
    }
  } else {
    float s[16], pl[16], rs[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      s[q] = src_ok ? st[src * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride +
                         (long long)q * cs]
                    : 0.0f;
      pl[q] = expf(P.log_poles[(long long)h * P.lp_stride_h + q * P.lp_stride_s]);
      rs[q] = P.residues[(long long)h * P.res_stride_h + q * P.res_stride_s];
    }
#pragma unroll
    for (int p = 0; p < DEC_MAXQ; ++p) {
      if (p < n) {
#pragma unroll
        for (int q = 0; q < 16; ++q) s[q] = add_rn(mul_rn(s[q], pl[q]), u[p]);
        if (dok[p]) {
#pragma unroll
          for (int q = 0; q < 16; ++q)
            st[dst[p] * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride +
               (long long)q * cs] = s[q];
        }
        y[p] = modal_readout16(s, rs);
      }
    }
  }

  // ---- output gate
  const bf16* Dg = static_cast<const bf16*>(P.D);
  const float d = Dg ? ldbf(Dg + h) : 0.0f;
#pragma unroll
  for (int p = 0; p < DEC_MAXQ; ++p) {
    if (p < n) {
      float yy = bf16r(y[p]);
      if (Dg) yy = bf16r(yy + bf16r(d * u[p]));
      out[(long long)(t0 + p) * A.ldo + h] = __float2bfloat16_rn(bf16r(xs[0][p] * yy));
    }
  }
}

int decode_launch(const hyena_layer_params& P, const hyena_decode_args& A, cudaStream_t st) {
  if (A.conv_state.cols > DEC_MAXW0)
    return fail(HYENA_ERR_UNSUPPORTED, "conv window wider than 8 columns");
  dim3 grid(A.num_reqs, (P.H + DEC_THREADS - 1) / DEC_THREADS);
  if (P.kind == HYENA_KIND_IIR) {
    if (P.K != 16) return fail(HYENA_ERR_UNSUPPORTED, "IIR decode supports modal order 16");
    decode_kernel<HYENA_KIND_IIR, 16><<<grid, DEC_THREADS, 0, st>>>(P, A);
  } else if (P.K == 128) {
    decode_kernel<HYENA_KIND_FIR, 128><<<grid, DEC_THREADS, 0, st>>>(P, A);
  } else if (P.K == 7) {
    decode_kernel<HYENA_KIND_FIR, 7><<<grid, DEC_THREADS, 0, st>>>(P, A);
  } else {
    return fail(HYENA_ERR_UNSUPPORTED, "FIR decode supports K = 7 or 128");
  }
  return check_launch("decode_kernel");
}

}  // namespace hb
