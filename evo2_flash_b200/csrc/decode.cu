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
constexpr int IIR_STAGE_MAXD = 20;  // widest S2 row (floats) the staged LI path handles

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

// V16 (LI only, chosen by the launcher): the staged state moves in 16-byte
// chunks; needs an odd row width and 16-byte-aligned blocks.
template <int KIND, int K, bool V16 = false>
__global__ void __launch_bounds__(DEC_THREADS)
decode_kernel(const hyena_layer_params P, const hyena_decode_args A) {
  pdl_entry();
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
  int accepted = A.accepted ? max(1, __ldg(A.accepted + r)) : 1;
  if (accepted > A.q) {  // past the slot table's columns
    if (threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_SEGMENT);
    accepted = A.q;
  }
  const int off = accepted - 1;
  const long long cin = __ldg(A.conv_in_block + (long long)r * A.conv_in_stride);
  const long long cout = __ldg(A.conv_out_block + (long long)r * A.conv_out_stride);
  bf16* out = static_cast<bf16*>(A.out);
  const bf16* z = static_cast<const bf16*>(A.z);

  if ((A.zero_null_rows && cin == A.null_block) || !block_ok(cin, A.conv_state)) {
    if (!block_ok(cin, A.conv_state) && threadIdx.x == 0)
      flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
    for (int p = 0; p < n; ++p) out[(long long)(t0 + p) * A.ldo + h] = __float2bfloat16_rn(0.0f);
    return;
  }

  // LI with contiguous modes: the warp's state run (32 channels x D floats of
  // the snapshot block) is put in flight now, into shared memory with
  // cp.async, and read after the short filter (see the staged path below).
  constexpr bool kIIR = KIND == HYENA_KIND_IIR;
  __shared__ __align__(16) float stage_sm[kIIR ? DEC_THREADS / 32 : 1]
                                        [kIIR ? 32 * (IIR_STAGE_MAXD + 1) : 1];
  const long long src = __ldg(A.in_slots + (long long)r * A.in_stride0 + (long long)off * A.in_stride1);
  const bool src_ok = block_ok(src, A.inner_state);
  const long long Dst = A.inner_state.dim_stride;
  const bool staged = kIIR && A.inner_state.col_stride == 1 && Dst >= 16 && Dst <= IIR_STAGE_MAXD;
  // odd row width (the stamp column makes 17): the shared-memory rows need no
  // padding, so the run moves as 16-byte chunks
  constexpr bool staged16 = V16;
  if constexpr (kIIR) {
    if (staged) {
      const int lane = threadIdx.x & 31;
      float* w = stage_sm[threadIdx.x >> 5];
      const int D = (int)Dst, pitch = D | 1;  // odd row pitch: conflict-free row reads
      const long long h0 = (long long)(h - lane);  // the warp's first channel
      const float* sp = static_cast<const float*>(A.inner_state.data) +
                        src * A.inner_state.block_stride + h0 * Dst;
      if (staged16) {  // 32 D floats = 8 D 16-byte chunks (h0 D is a multiple of 4)
        for (int j = lane; j < 8 * D; j += 32) {
          if (src_ok)
            cp_async16(&w[4 * j], sp + 4 * j);
          else
            *reinterpret_cast<float4*>(&w[4 * j]) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      } else {
        for (int j = lane; j < 32 * D; j += 32) {
          float* d = &w[(j / D) * pitch + j % D];
          if (src_ok)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                             static_cast<uint32_t>(__cvta_generic_to_shared(d))),
                         "l"(sp + j)
                         : "memory");
          else
            *d = 0.0f;
        }
      }
      cp_async_commit();
    }
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
  long long dst[DEC_MAXQ];
  bool dok[DEC_MAXQ];
#pragma unroll
  for (int p = 0; p < DEC_MAXQ; ++p) {
    dst[p] = p < n ? __ldg(A.out_slots + (long long)r * A.out_stride0 + (long long)p * A.out_stride1) : 0;
    dok[p] = p < n && block_ok(dst[p], A.inner_state) &&
             !(A.skip_null_writes && dst[p] == A.null_block);
  }
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
    if constexpr (V16) {  // contiguous, 16-byte-aligned rows (checked by the launcher)
      const float4* lp4 = reinterpret_cast<const float4*>(P.log_poles + (long long)h * P.lp_stride_h);
      const float4* rs4 = reinterpret_cast<const float4*>(P.residues + (long long)h * P.res_stride_h);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const float4 a = __ldg(lp4 + q4), b = __ldg(rs4 + q4);
        pl[4 * q4] = expf(a.x); pl[4 * q4 + 1] = expf(a.y);
        pl[4 * q4 + 2] = expf(a.z); pl[4 * q4 + 3] = expf(a.w);
        rs[4 * q4] = b.x; rs[4 * q4 + 1] = b.y; rs[4 * q4 + 2] = b.z; rs[4 * q4 + 3] = b.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        pl[q] = expf(P.log_poles[(long long)h * P.lp_stride_h + q * P.lp_stride_s]);
        rs[q] = P.residues[(long long)h * P.res_stride_h + q * P.res_stride_s];
      }
    }
    // Modes contiguous (S2 rows of D >= 16 floats, the stamp column included):
    // a warp's 32 channels are one contiguous run of 32 D floats per block, so
    // the state and every snapshot move through shared memory with coalesced
    // 4-byte accesses (the stamp column is never written) instead of 16
    // scattered ones per thread.
    const long long D = Dst;
    if (staged) {
      const int lane = threadIdx.x & 31;
      float* w = stage_sm[threadIdx.x >> 5];
      const long long h0 = (long long)(h - lane);  // the warp's first channel
      const int pitch = (int)(D | 1);
      const int run = 32 * (int)D;
      cp_async_wait<0>();  // the state run put in flight before the short filter
      __syncwarp();
#pragma unroll
      for (int q = 0; q < 16; ++q) s[q] = w[lane * pitch + q];
#pragma unroll
      for (int p = 0; p < DEC_MAXQ; ++p) {
        if (p < n) {  // n and dok[p] are per request: uniform in the warp
#pragma unroll
          for (int q = 0; q < 16; ++q) s[q] = add_rn(mul_rn(s[q], pl[q]), u[p]);
          if (dok[p]) {
            float* dp = st + dst[p] * A.inner_state.block_stride + h0 * D;
            __syncwarp();  // the previous snapshot's stores have read the buffer
#pragma unroll
            for (int q = 0; q < 16; ++q) w[lane * pitch + q] = s[q];
            if (staged16) {
              // the columns past the 16 modes (the position stamp) keep the
              // destination block's values: read them into the run first
              for (int c = 16; c < (int)D; ++c) w[lane * pitch + c] = dp[(long long)lane * D + c];
              __syncwarp();
              for (int j = lane; j < 8 * (int)D; j += 32)
                *reinterpret_cast<float4*>(dp + 4 * j) = *reinterpret_cast<const float4*>(&w[4 * j]);
            } else {
              __syncwarp();
              for (int j = lane; j < run; j += 32) {
                const int c = j % (int)D;
                if (c < 16) dp[j] = w[(j / (int)D) * pitch + c];
              }
            }
          }
          y[p] = modal_readout16(s, rs);
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 16; ++q)
        s[q] = src_ok ? st[src * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride +
                           (long long)q * cs]
                      : 0.0f;
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

// ---------------------------------------------------------------- q = 1 fast path
// Ordinary decode (one token per request, accepted = 1, a 2-column short window
// with unit channel stride): a thread owns 4 consecutive channels (FIR) or one
// channel's 16 modes (IIR) and streams its state with 16-byte accesses, 16 taps in
// flight.  Same arithmetic, order and rounding as decode_kernel.  The verify
// kernels use blocks of FAST_THREADS, the one-token FIR kernel blocks of
// Q1_THREADS (64: 1.1 us faster per decode step of the 7B triple at 128
// requests than 128; 64 made the verify step 0.507 -> 0.530 ms).
constexpr int FAST_THREADS = 128;
constexpr int Q1_THREADS = 64;

__device__ __forceinline__ void load_bf16x4(const bf16* p, float (&v)[4]) {
  const uint2 r = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&r.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&r.y);
  v[0] = __low2float(a); v[1] = __high2float(a); v[2] = __low2float(b); v[3] = __high2float(b);
}

__device__ __forceinline__ void store_bf16x4(bf16* p, const float (&v)[4]) {
  uint2 r;
  const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
  const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
  r.x = *reinterpret_cast<const uint32_t*>(&a);
  r.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = r;
}

// The K=3 short filter of 4 consecutive channels' triples: their 12 z columns
// as 6 bf16x2 column pairs (2j, 2j+1) through short_tap2, which rounds each
// product to bf16 and sums oldest first in fp32 exactly as short_tap does.
struct Taps4 {
  bf162 w[6][3];  // tap k of column pair j
};
// From the 36 contiguous short taps of the 4 channels (tap e = 3 col + k sits
// in word e / 2, half e % 2).
__device__ __forceinline__ Taps4 taps4(const uint2 (&swr)[9]) {
  auto word = [&](int i) -> uint32_t { return (i & 1) ? swr[i >> 1].y : swr[i >> 1].x; };
  Taps4 T;
#pragma unroll
  for (int j = 0; j < 6; ++j)
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int e1 = 6 * j + k, e2 = 6 * j + 3 + k;
      const uint32_t sel = ((e1 & 1) ? 0x0032u : 0x0010u) | ((e2 & 1) ? 0x7600u : 0x5400u);
      T.w[j][k] = as_bf162(__byte_perm(word(e1 >> 1), word(e2 >> 1), sel));
    }
  return T;
}
// o = the filter outputs of one row x from the window rows c0 (older) and c1.
__device__ __forceinline__ void short4(const Taps4& T, const uint32_t (&c0)[6],
                                       const uint32_t (&c1)[6], const uint32_t (&x)[6],
                                       uint32_t (&o)[6]) {
#pragma unroll
  for (int j = 0; j < 6; ++j)
    o[j] = as_u32(short_tap2(as_bf162(c0[j]), as_bf162(c1[j]), as_bf162(x[j]), T.w[j][0],
                             T.w[j][1], T.w[j][2]));
}
// Channel c's (x2, x1, v) are columns 3c .. 3c+2: words (w0, w1, w2) of channels
// (0, 1) hold (x2_0, x1_0), (v_0, x2_1), (x1_1, v_1); likewise (w3, w4, w5) for
// channels (2, 3).  u = bf16(x1 v) is one bf16x2 product (exact product, one
// rounding: bf16r(x1 * v)).
__device__ __forceinline__ void split4(const uint32_t (&o)[6], float (&x2)[4], float (&u)[4]) {
#pragma unroll
  for (int hp = 0; hp < 2; ++hp) {
    const uint32_t w0 = o[3 * hp], w1 = o[3 * hp + 1], w2 = o[3 * hp + 2];
    const float2 a = __bfloat1622float2(as_bf162(__byte_perm(w0, w1, 0x7610)));
    const float2 b = __bfloat1622float2(__hmul2(as_bf162(__byte_perm(w0, w2, 0x5432)),
                                                as_bf162(__byte_perm(w1, w2, 0x7610))));
    x2[2 * hp] = a.x;
    x2[2 * hp + 1] = a.y;
    u[2 * hp] = b.x;
    u[2 * hp + 1] = b.y;
  }
}

// Short filter + gate for `C` consecutive channels starting at h, in two
// halves so that callers can put its loads in flight together with their own:
// gate_load reads the triple row of z, window columns 0, 1 of S0 (block cin)
// and the short taps; gate_finish computes x2 and u per channel and writes
// [c1, x] to block cout.
template <int C>
struct GateIn {
  float zx[3 * C], w0[3 * C], w1[3 * C];
  uint2 swr[9 * C / 4];  // short taps of the C channels: 9C contiguous bf16
};

template <int C>
__device__ __forceinline__ void gate_load(const hyena_layer_params& P, const hyena_decode_args& A,
                                          int t0, int h, long long cin, GateIn<C>& g) {
  static_assert(C % 4 == 0, "vector path: 4-channel multiples");
  const bf16* z = static_cast<const bf16*>(A.z) + (long long)t0 * A.ldz + 3 * h;
  const bf16* s0 = static_cast<const bf16*>(A.conv_state.data);
  const bf16* c0p = s0 + cin * A.conv_state.block_stride + 3 * h;
  const bf16* c1p = c0p + A.conv_state.col_stride;
  const uint2* swv = reinterpret_cast<const uint2*>(static_cast<const bf16*>(P.short_w) + 9 * h);
#pragma unroll
  for (int i = 0; i < 9 * C / 4; ++i) g.swr[i] = __ldg(swv + i);
#pragma unroll
  for (int i = 0; i < 3 * C; i += 4) {
    float a[4], b[4];
    load_bf16x4(z + i, a);
#pragma unroll
    for (int k = 0; k < 4; ++k) g.zx[i + k] = a[k];
    load_bf16x4(c0p + i, a);
    load_bf16x4(c1p + i, b);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      g.w0[i + k] = a[k];
      g.w1[i + k] = b[k];
    }
  }
}

template <int C>
__device__ __forceinline__ void gate_finish(const hyena_decode_args& A, int h, long long cout,
                                            bool write_conv, const GateIn<C>& g, float (&x2)[C],
                                            float (&u)[C]) {
  const bf16* sw = reinterpret_cast<const bf16*>(g.swr);
  float o[3 * C];
#pragma unroll
  for (int i = 0; i < 3 * C; ++i)
    o[i] = short_tap(g.w0[i], g.w1[i], g.zx[i], __bfloat162float(sw[3 * i]),
                     __bfloat162float(sw[3 * i + 1]), __bfloat162float(sw[3 * i + 2]));
  if (write_conv) {
    bf16* s0 = static_cast<bf16*>(A.conv_state.data);
    bf16* d0 = s0 + cout * A.conv_state.block_stride + 3 * h;
    bf16* d1 = d0 + A.conv_state.col_stride;
#pragma unroll
    for (int i = 0; i < 3 * C; i += 4) {
      float a[4] = {g.w1[i], g.w1[i + 1], g.w1[i + 2], g.w1[i + 3]};
      float b[4] = {g.zx[i], g.zx[i + 1], g.zx[i + 2], g.zx[i + 3]};
      store_bf16x4(d0 + i, a);
      store_bf16x4(d1 + i, b);
    }
  }
#pragma unroll
  for (int c = 0; c < C; ++c) {
    x2[c] = o[3 * c];
    u[c] = bf16r(o[3 * c + 1] * o[3 * c + 2]);
  }
}

template <int K>
__global__ void __launch_bounds__(Q1_THREADS)
decode_fir_q1_kernel(const hyena_layer_params P, const hyena_decode_args A) {
  pdl_entry();
  constexpr int HIST = K - 1;
  constexpr int U = 8;  // taps in flight
  const int r = blockIdx.x;
  const int h = 4 * (blockIdx.y * Q1_THREADS + threadIdx.x);
  if (h >= P.H) return;
  // Routing first, all four loads in flight at once.
  const long long cin = __ldg(A.conv_in_block + (long long)r * A.conv_in_stride);
  const long long cout = __ldg(A.conv_out_block + (long long)r * A.conv_out_stride);
  const long long src = __ldg(A.in_slots + (long long)r * A.in_stride0);
  const long long dst = __ldg(A.out_slots + (long long)r * A.out_stride0);
  bf16* out = static_cast<bf16*>(A.out) + (long long)r * A.ldo + h;
  if ((A.zero_null_rows && cin == A.null_block) || !block_ok(cin, A.conv_state)) {
    if (!block_ok(cin, A.conv_state) && threadIdx.x == 0)
      flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    store_bf16x4(out, zero);
    return;
  }
  const bool write_conv = block_ok(cout, A.conv_state) &&
                          !(A.skip_null_writes && cout == A.null_block);
  // The gate's inputs are loaded now; for the long window they are consumed
  // after the window stream, so that both sets of loads are in flight at once.
  GateIn<4> gin;
  gate_load<4>(P, A, r, h, cin, gin);
  float x2[4], u[4];
  if constexpr (HIST < 32) gate_finish<4>(A, h, cout, write_conv, gin, x2, u);  // short window
  const bool src_ok = block_ok(src, A.inner_state);
  const bool dok = block_ok(dst, A.inner_state) && !(A.skip_null_writes && dst == A.null_block);
  if (!src_ok && threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
  float* st = static_cast<float*>(A.inner_state.data);
  const long long cs = A.inner_state.col_stride;
  const float* sp = st + (src_ok ? src : 0) * A.inner_state.block_stride + h;
  float* dp = st + (dok ? dst : 0) * A.inner_state.block_stride + h;
  const bf16* w = static_cast<const bf16*>(P.inner_w) + h;  // (K, H) layout, unit channel stride
  const long long wk = P.inner_w_stride_k;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int k0 = 0; k0 < HIST; k0 += U) {
    float4 sv[U];
    uint2 wr[U];
#pragma unroll
    for (int t = 0; t < U; ++t) {
      if (k0 + t < HIST) {
        sv[t] = src_ok ? *reinterpret_cast<const float4*>(sp + (long long)(k0 + t) * cs)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        wr[t] = __ldg(reinterpret_cast<const uint2*>(w + (long long)(k0 + t) * wk));
      }
    }
#pragma unroll
    for (int t = 0; t < U; ++t) {
      if (k0 + t < HIST) {
        const float2 wa = __bfloat1622float2(as_bf162(wr[t].x));
        const float2 wb = __bfloat1622float2(as_bf162(wr[t].y));
        acc[0] = fmaf(wa.x, sv[t].x, acc[0]);
        acc[1] = fmaf(wa.y, sv[t].y, acc[1]);
        acc[2] = fmaf(wb.x, sv[t].z, acc[2]);
        acc[3] = fmaf(wb.y, sv[t].w, acc[3]);
        if (dok && k0 + t >= 1) *reinterpret_cast<float4*>(dp + (long long)(k0 + t - 1) * cs) = sv[t];
      }
    }
  }
  if constexpr (HIST >= 32) gate_finish<4>(A, h, cout, write_conv, gin, x2, u);
  float wl[4];
  load_bf16x4(w + (long long)HIST * wk, wl);
#pragma unroll
  for (int c = 0; c < 4; ++c) acc[c] = fmaf(wl[c], u[c], acc[c]);
  if (dok) *reinterpret_cast<float4*>(dp + (long long)(HIST - 1) * cs) = make_float4(u[0], u[1], u[2], u[3]);
  const bf16* Dg = static_cast<const bf16*>(P.D);
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  if (Dg) load_bf16x4(Dg + h, d);
  float g[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float yy = bf16r(acc[c]);
    if (Dg) yy = bf16r(yy + bf16r(d[c] * u[c]));
    g[c] = bf16r(x2[c] * yy);
  }
  store_bf16x4(out, g);
}

// LI q = 1 decode, one lane per channel for LQ_R requests: a block holds
// LQ_THREADS consecutive channels and needs no barrier, so its warps run
// independently (64-lane blocks: 0.6 us faster per decode step than 128 or
// 256; two requests per lane instead of four: 1.7 us slower).
// A lane computes its channel's exp(log-pole)s and loads its residues, short
// taps and D once for all its requests; it then walks the requests with the
// next request's state row (16-byte loads), z triple and window columns in
// flight while the current one is computed: the K=3 filter of the triple
// (short_tap, the arithmetic of decode_kernel), the 16 modes advanced in packed
// f32x2 arithmetic (same roundings), the row and the shifted window written
// back, modal_readout16's halving tree.
constexpr int LQ_THREADS = 64;
constexpr int LQ_R = 4;

struct LqIn {
  float4 sv[4];                // the 16-mode row
  bf16 z[3], c0[3], c1[3];     // z triple, window columns 0 and 1
};

__global__ void __launch_bounds__(LQ_THREADS)
decode_iir_q1_lane_kernel(const hyena_layer_params P, const hyena_decode_args A) {
  pdl_entry();
  const int r0 = blockIdx.x * LQ_R;
  const int h = blockIdx.y * LQ_THREADS + threadIdx.x;
  if (h >= P.H) return;
  const int nr = min(LQ_R, A.num_reqs - r0);
  // routing of the lane's requests, all loads at once
  long long cin[LQ_R], cout[LQ_R], src[LQ_R], dst[LQ_R];
#pragma unroll
  for (int i = 0; i < LQ_R; ++i) {
    cin[i] = cout[i] = src[i] = dst[i] = -1;
    if (i < nr) {
      const int r = r0 + i;
      cin[i] = __ldg(A.conv_in_block + (long long)r * A.conv_in_stride);
      cout[i] = __ldg(A.conv_out_block + (long long)r * A.conv_out_stride);
      src[i] = __ldg(A.in_slots + (long long)r * A.in_stride0);
      dst[i] = __ldg(A.out_slots + (long long)r * A.out_stride0);
    }
  }
  float* st = static_cast<float*>(A.inner_state.data);
  const long long D = A.inner_state.dim_stride;
  const bf16* s0 = static_cast<const bf16*>(A.conv_state.data);
  auto zero_row = [&](int i) {
    return (A.zero_null_rows && cin[i] == A.null_block) || !block_ok(cin[i], A.conv_state);
  };
  auto load = [&](int i, LqIn& in) {
#pragma unroll
    for (int k = 0; k < 4; ++k) in.sv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (zero_row(i)) return;
    if (block_ok(src[i], A.inner_state)) {
      const float4* sp = reinterpret_cast<const float4*>(st + src[i] * A.inner_state.block_stride + h * D);
#pragma unroll
      for (int k = 0; k < 4; ++k) in.sv[k] = sp[k];
    }
    const bf16* zr = static_cast<const bf16*>(A.z) + (long long)(r0 + i) * A.ldz + 3 * h;
    const bf16* w0p = s0 + cin[i] * A.conv_state.block_stride + 3 * h;
    const bf16* w1p = w0p + A.conv_state.col_stride;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      in.z[j] = zr[j];
      in.c0[j] = w0p[j];
      in.c1[j] = w1p[j];
    }
  };
  LqIn cur;
  load(0, cur);
  // per-channel parameters, once for all requests
  float w[9];
  const bf16* swp = static_cast<const bf16*>(P.short_w) + 9 * h;
#pragma unroll
  for (int j = 0; j < 9; ++j) w[j] = __bfloat162float(__ldg(swp + j));
  const float4* lp4 = reinterpret_cast<const float4*>(P.log_poles + (long long)h * P.lp_stride_h);
  const float4* rs4 = reinterpret_cast<const float4*>(P.residues + (long long)h * P.res_stride_h);
  float2 pl2[8], rs2[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float4 a = __ldg(lp4 + k), b = __ldg(rs4 + k);
    pl2[2 * k] = make_float2(expf(a.x), expf(a.y));
    pl2[2 * k + 1] = make_float2(expf(a.z), expf(a.w));
    rs2[2 * k] = make_float2(b.x, b.y);
    rs2[2 * k + 1] = make_float2(b.z, b.w);
  }
  const bf16* Dg = static_cast<const bf16*>(P.D);
  const float dval = Dg ? ldbf(Dg + h) : 0.0f;

#pragma unroll
  for (int i = 0; i < LQ_R; ++i) {
    if (i >= nr) break;
    LqIn nxt;
    if (i + 1 < nr) load(i + 1, nxt);
    bf16* out = static_cast<bf16*>(A.out) + (long long)(r0 + i) * A.ldo + h;
    if (zero_row(i)) {
      if (!block_ok(cin[i], A.conv_state) && threadIdx.x == 0)
        flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
      *out = __float2bfloat16_rn(0.0f);
    } else {
      if (!block_ok(src[i], A.inner_state) && threadIdx.x == 0)
        flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
      float o[3];
#pragma unroll
      for (int j = 0; j < 3; ++j)
        o[j] = short_tap(__bfloat162float(cur.c0[j]), __bfloat162float(cur.c1[j]),
                         __bfloat162float(cur.z[j]), w[3 * j], w[3 * j + 1], w[3 * j + 2]);
      const float x2 = o[0];
      const float u = bf16r(o[1] * o[2]);
      if (block_ok(cout[i], A.conv_state) && !(A.skip_null_writes && cout[i] == A.null_block)) {
        bf16* d0 = static_cast<bf16*>(A.conv_state.data) + cout[i] * A.conv_state.block_stride + 3 * h;
        bf16* d1 = d0 + A.conv_state.col_stride;
#pragma unroll
        for (int j = 0; j < 3; ++j) {  // window <- [old column 1, this row]
          d0[j] = cur.c1[j];
          d1[j] = cur.z[j];
        }
      }
      float2 s2[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s2[2 * k] = make_float2(cur.sv[k].x, cur.sv[k].y);
        s2[2 * k + 1] = make_float2(cur.sv[k].z, cur.sv[k].w);
      }
      const float2 u2 = make_float2(u, u);
#pragma unroll
      for (int k = 0; k < 8; ++k) s2[k] = fadd2(fmul2(s2[k], pl2[k]), u2);  // s p + u, no FMA
      if (block_ok(dst[i], A.inner_state) && !(A.skip_null_writes && dst[i] == A.null_block)) {
        float4* dp = reinterpret_cast<float4*>(st + dst[i] * A.inner_state.block_stride + h * D);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          dp[k] = make_float4(s2[2 * k].x, s2[2 * k].y, s2[2 * k + 1].x, s2[2 * k + 1].y);
      }
      float y = bf16r(modal_readout16_x2(s2, rs2));
      if (Dg) y = bf16r(y + bf16r(dval * u));
      *out = __float2bfloat16_rn(bf16r(x2 * y));
    }
    if (i + 1 < nr) cur = nxt;
  }
}

static bool aligned_elems(const void* p, int64_t stride_elems, int elem_bytes, int vec_bytes) {
  return (reinterpret_cast<uintptr_t>(p) % vec_bytes) == 0 &&
         (stride_elems * elem_bytes) % vec_bytes == 0;
}

// The q = 1 kernels apply when each request has exactly one token, no accepted
// offsets, a 2-column short window, unit channel strides and 16-byte-aligned rows.
static bool fast_path_ok(const hyena_layer_params& P, const hyena_decode_args& A) {
  if (A.q != 1 || A.token_start != nullptr || A.accepted != nullptr) return false;
  if (A.conv_state.cols != 2 || A.conv_state.dim_stride != 1) return false;
  if (!aligned_elems(A.z, A.ldz, 2, 8) || !aligned_elems(A.out, A.ldo, 2, 8)) return false;
  if (!aligned_elems(P.short_w, 0, 2, 8)) return false;
  if (!aligned_elems(A.conv_state.data, A.conv_state.block_stride, 2, 8) ||
      (A.conv_state.col_stride * 2) % 8 != 0)
    return false;
  const hyena_state_view& s = A.inner_state;
  if (P.kind == HYENA_KIND_FIR) {
    if (s.dim_stride != 1 || P.inner_w_stride_h != 1 || (P.inner_w_stride_k * 2) % 8 != 0) return false;
    if (!aligned_elems(P.inner_w, 0, 2, 8) || (P.D && !aligned_elems(P.D, 0, 2, 8))) return false;
    return aligned_elems(s.data, s.block_stride, 4, 16) && (s.col_stride * 4) % 16 == 0 &&
           P.H % 4 == 0;
  }
  return s.col_stride == 1 && aligned_elems(s.data, s.block_stride, 4, 16) &&
         (s.dim_stride * 4) % 16 == 0 && P.lp_stride_s == 1 && P.res_stride_s == 1 &&
         aligned_elems(P.log_poles, P.lp_stride_h, 4, 16) &&
         aligned_elems(P.residues, P.res_stride_h, 4, 16) && P.H % 4 == 0;
}

// The short filter of one verify step for 4 channels, whose (x2, x1, v) triples
// are 12 contiguous bf16 columns: window columns off, off + 1 of S0 block cin,
// then the n verified rows of z, oldest first (short_tap per column, the
// arithmetic of decode_kernel); x2 and u = bf16(x1 v) per position.  The S0
// window of block cout becomes old columns off + 1 .. followed by the new rows,
// column by column in ascending order, so that in place (cout == cin) each old
// column is read before it is overwritten.  Every access moves 4 bf16 (8 bytes).
template <int NQ>
__device__ __forceinline__ void verify_gate4(const hyena_layer_params& P, const hyena_decode_args& A,
                                             int h, int t0, int n, int off, long long cin,
                                             long long cout, bool write_conv,
                                             float (&x2v)[NQ][4], float (&uv)[NQ][4]) {
  const int W0 = A.conv_state.cols;
  bf16* s0 = static_cast<bf16*>(A.conv_state.data);
  const long long bs = A.conv_state.block_stride, cs = A.conv_state.col_stride;
  const bf16* win = s0 + cin * bs + 3 * h;
  const uint2* swv = reinterpret_cast<const uint2*>(static_cast<const bf16*>(P.short_w) + 9 * h);
  uint2 swr[9];  // 36 taps: column j's three at 3j
#pragma unroll
  for (int i = 0; i < 9; ++i) swr[i] = __ldg(swv + i);
  const Taps4 T = taps4(swr);
  uint32_t c0[6], c1[6];  // window columns off, off + 1 as column-pair words
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    uint2 a = make_uint2(0u, 0u), b = make_uint2(0u, 0u);
    if (off < W0) a = *reinterpret_cast<const uint2*>(win + (long long)off * cs + 4 * i);
    if (off + 1 < W0) b = *reinterpret_cast<const uint2*>(win + (long long)(off + 1) * cs + 4 * i);
    c0[2 * i] = a.x; c0[2 * i + 1] = a.y;
    c1[2 * i] = b.x; c1[2 * i + 1] = b.y;
  }
  const bf16* z = static_cast<const bf16*>(A.z);
#pragma unroll
  for (int p = 0; p < NQ; ++p) {
#pragma unroll
    for (int c = 0; c < 4; ++c) x2v[p][c] = uv[p][c] = 0.0f;
    if (p < n) {
      const uint2* zp = reinterpret_cast<const uint2*>(z + (long long)(t0 + p) * A.ldz + 3 * h);
      uint32_t xw[6], o[6];
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        const uint2 zw = zp[i];
        xw[2 * i] = zw.x;
        xw[2 * i + 1] = zw.y;
      }
      short4(T, c0, c1, xw, o);
#pragma unroll
      for (int j = 0; j < 6; ++j) {
        c0[j] = c1[j];
        c1[j] = xw[j];
      }
      split4(o, x2v[p], uv[p]);
    }
  }
  if (write_conv) {
    // every value of the new window is loaded before the first store, so the
    // loads overlap and, in place, each old column is read before it is
    // overwritten
    bf16* wout = s0 + cout * bs + 3 * h;
    const int val = W0 - n;  // columns kept from the old window
    uint2 v[DEC_MAXW0][3];
#pragma unroll
    for (int i = 0; i < DEC_MAXW0; ++i) {
#pragma unroll
      for (int k = 0; k < 3; ++k) v[i][k] = make_uint2(0u, 0u);
      if (i < W0) {
        const uint2* sp = nullptr;
        if (i < val) {
          const int sc = off + 1 + i;
          if (sc < W0) sp = reinterpret_cast<const uint2*>(win + (long long)sc * cs);
        } else {  // the verified row i - val again (an L1 hit)
          sp = reinterpret_cast<const uint2*>(z + (long long)(t0 + i - val) * A.ldz + 3 * h);
        }
        if (sp) {
#pragma unroll
          for (int k = 0; k < 3; ++k) v[i][k] = sp[k];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < DEC_MAXW0; ++i) {
      if (i < W0) {
        uint2* dp = reinterpret_cast<uint2*>(wout + (long long)i * cs);
#pragma unroll
        for (int k = 0; k < 3; ++k) dp[k] = v[i][k];
      }
    }
  }
}

// FIR verify (q <= VQ positions per request, speculative windows): one thread
// per (request, 4 channels).  The short filter runs per column exactly as in
// decode_kernel; the inner FIR streams the accepted snapshot once with 16-byte
// loads (4 channels), keeps the last VQ taps' weights in registers, and writes
// every verifier snapshot with 16-byte stores.  Same arithmetic and order as
// decode_kernel (fp32 FMA over taps oldest first, then the verified tokens).
constexpr int VQ = 4;

template <int K>
__global__ void __launch_bounds__(FAST_THREADS, 4)
decode_fir_verify_kernel(const hyena_layer_params P, const hyena_decode_args A) {
  pdl_entry();
  constexpr int HIST = K - 1;
  constexpr int U = 6;  // window columns in flight
  const int r = blockIdx.x;
  const int h = 4 * (blockIdx.y * FAST_THREADS + threadIdx.x);
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
  if (n > A.q || n > VQ) {
    if (threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_SEGMENT);
    n = min(A.q, VQ);
  }
  int accepted = A.accepted ? max(1, __ldg(A.accepted + r)) : 1;
  if (accepted > A.q) {  // past the slot table's columns
    if (threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_SEGMENT);
    accepted = A.q;
  }
  const int off = accepted - 1;
  const long long cin = __ldg(A.conv_in_block + (long long)r * A.conv_in_stride);
  const long long cout = __ldg(A.conv_out_block + (long long)r * A.conv_out_stride);
  const long long src = __ldg(A.in_slots + (long long)r * A.in_stride0 + (long long)off * A.in_stride1);
  long long dst[VQ];
  bool dok[VQ];
#pragma unroll
  for (int p = 0; p < VQ; ++p) {
    dst[p] = p < n ? __ldg(A.out_slots + (long long)r * A.out_stride0 + (long long)p * A.out_stride1) : 0;
    dok[p] = p < n && block_ok(dst[p], A.inner_state) &&
             !(A.skip_null_writes && dst[p] == A.null_block);
  }
  bf16* out = static_cast<bf16*>(A.out);
  if ((A.zero_null_rows && cin == A.null_block) || !block_ok(cin, A.conv_state)) {
    if (!block_ok(cin, A.conv_state) && threadIdx.x == 0)
      flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < n; ++p) store_bf16x4(out + (long long)(t0 + p) * A.ldo + h, zero);
    return;
  }
  const bool src_ok = block_ok(src, A.inner_state);
  if (!src_ok && threadIdx.x == 0) flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
  float* st = static_cast<float*>(A.inner_state.data);
  const long long cs = A.inner_state.col_stride;
  const float* sp = st + (src_ok ? src : 0) * A.inner_state.block_stride + h;
  float4 sv[U];
#pragma unroll
  for (int t = 0; t < U; ++t)
    sv[t] = (src_ok && t < HIST) ? *reinterpret_cast<const float4*>(sp + (long long)t * cs)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);

  // ---- inner FIR over the accepted snapshot, verifier snapshots written
  const bf16* w = static_cast<const bf16*>(P.inner_w) + h;  // (K, H), unit channel stride
  const long long wk = P.inner_w_stride_k;
  float y[VQ][4];
#pragma unroll
  for (int p = 0; p < VQ; ++p)
#pragma unroll
    for (int c = 0; c < 4; ++c) y[p][c] = 0.0f;
  float wr[VQ][4];  // wr[j] = weights of tap k - j
#pragma unroll
  for (int j = 0; j < VQ; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) wr[j][c] = 0.0f;
  float* dbase[VQ];
#pragma unroll
  for (int p = 0; p < VQ; ++p) dbase[p] = st + (dok[p] ? dst[p] : 0) * A.inner_state.block_stride + h;
  // the taps of a chunk are loaded with its window columns, a chunk ahead
  // (read-only loads: nothing orders them after the snapshot stores)
  uint2 wc[U];
#pragma unroll
  for (int t = 0; t < U; ++t)
    wc[t] = t < HIST ? __ldg(reinterpret_cast<const uint2*>(w + (long long)t * wk)) : make_uint2(0u, 0u);
#pragma unroll 1
  for (int k0 = 0; k0 < HIST; k0 += U) {
    float4 nx[U];
    uint2 wn[U];
#pragma unroll
    for (int t = 0; t < U; ++t) {
      nx[t] = (src_ok && k0 + U + t < HIST)
                  ? *reinterpret_cast<const float4*>(sp + (long long)(k0 + U + t) * cs)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
      wn[t] = k0 + U + t < HIST ? __ldg(reinterpret_cast<const uint2*>(w + (long long)(k0 + U + t) * wk))
                                : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int t = 0; t < U; ++t) {
      const int k = k0 + t;
      if (k < HIST) {
#pragma unroll
        for (int j = VQ - 1; j > 0; --j)
#pragma unroll
          for (int c = 0; c < 4; ++c) wr[j][c] = wr[j - 1][c];
        {
          const float2 a = __bfloat1622float2(as_bf162(wc[t].x));
          const float2 b = __bfloat1622float2(as_bf162(wc[t].y));
          wr[0][0] = a.x; wr[0][1] = a.y; wr[0][2] = b.x; wr[0][3] = b.y;
        }
        const float sx[4] = {sv[t].x, sv[t].y, sv[t].z, sv[t].w};
#pragma unroll
        for (int p = 0; p < VQ; ++p) {
          if (p < n && k >= p) {
#pragma unroll
            for (int c = 0; c < 4; ++c) y[p][c] = fmaf(wr[p][c], sx[c], y[p][c]);
          }
          if (p < n && dok[p] && k - p - 1 >= 0)
            *reinterpret_cast<float4*>(dbase[p] + (long long)(k - p - 1) * cs) = sv[t];
        }
      }
    }
#pragma unroll
    for (int t = 0; t < U; ++t) {
      sv[t] = nx[t];
      wc[t] = wn[t];
    }
  }
  // ---- short filter of the 4 channels' triples, window shift (after the
  // stream, so that its values are not held in registers across it)
  const bool write_conv = block_ok(cout, A.conv_state) &&
                          !(A.skip_null_writes && cout == A.null_block);
  float x2v[VQ][4], uv[VQ][4];
  verify_gate4<VQ>(P, A, h, t0, n, off, cin, cout, write_conv, x2v, uv);

  // the verified tokens themselves: newest taps, and the tail of each snapshot
#pragma unroll
  for (int p = 0; p < VQ; ++p) {
    if (p < n) {
#pragma unroll
      for (int i = 0; i < VQ; ++i) {
        if (i < p) {
          float wv[4];
          load_bf16x4(w + (long long)(HIST + i - p) * wk, wv);
#pragma unroll
          for (int c = 0; c < 4; ++c) y[p][c] = fmaf(wv[c], uv[i][c], y[p][c]);
        }
      }
      float wl[4];
      load_bf16x4(w + (long long)HIST * wk, wl);
#pragma unroll
      for (int c = 0; c < 4; ++c) y[p][c] = fmaf(wl[c], uv[p][c], y[p][c]);
      if (dok[p]) {
#pragma unroll
        for (int m = 0; m < VQ; ++m)
          if (m <= p)
            *reinterpret_cast<float4*>(dbase[p] + (long long)(HIST - 1 - p + m) * cs) =
                make_float4(uv[m][0], uv[m][1], uv[m][2], uv[m][3]);
      }
    }
  }
  // ---- output gate
  const bf16* Dg = static_cast<const bf16*>(P.D);
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  if (Dg) load_bf16x4(Dg + h, d);
#pragma unroll
  for (int p = 0; p < VQ; ++p) {
    if (p < n) {
      float g[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float yy = bf16r(y[p][c]);
        if (Dg) yy = bf16r(yy + bf16r(d[c] * uv[p][c]));
        g[c] = bf16r(x2v[p][c] * yy);
      }
      store_bf16x4(out + (long long)(t0 + p) * A.ldo + h, g);
    }
  }
}

// verify_gate4 and the 4-channel output stores: 8-byte accesses to z, the
// short taps, the S0 window (unit channel stride) and out, and to D.
static bool gate4_ok(const hyena_layer_params& P, const hyena_decode_args& A) {
  if (A.q > VQ || A.conv_state.dim_stride != 1) return false;
  if (!aligned_elems(A.z, A.ldz, 2, 8) || !aligned_elems(P.short_w, 0, 2, 8)) return false;
  if (!aligned_elems(A.conv_state.data, A.conv_state.block_stride, 2, 8) ||
      (A.conv_state.col_stride * 2) % 8 != 0)
    return false;
  if (P.D && !aligned_elems(P.D, 0, 2, 8)) return false;
  return aligned_elems(A.out, A.ldo, 2, 8) && P.H % 4 == 0;
}

// The FIR verify path: up to VQ positions, unit channel strides, 16-byte rows.
static bool fir_verify_ok(const hyena_layer_params& P, const hyena_decode_args& A) {
  if (P.kind != HYENA_KIND_FIR || !gate4_ok(P, A)) return false;
  const hyena_state_view& s = A.inner_state;
  if (s.dim_stride != 1 || P.inner_w_stride_h != 1 || (P.inner_w_stride_k * 2) % 8 != 0) return false;
  if (!aligned_elems(P.inner_w, 0, 2, 8) || (P.D && !aligned_elems(P.D, 0, 2, 8))) return false;
  return aligned_elems(s.data, s.block_stride, 4, 16) && (s.col_stride * 4) % 16 == 0 &&
         P.H % 4 == 0;
}

// LI verify (q <= VQ positions per request, speculative windows, S2 rows of
// D = 16 .. 20 floats: the 16 modes, then padding columns, the last of channel
// 0 holding the block's position stamp).  Every warp works on its own, with no
// block barrier: 32 channels (one per lane) of LW_R requests, whose rows form
// one contiguous, 16-byte-aligned run of 32 D floats per state block.
//   1. lanes 0 .. LW_R-1 resolve one request each (every routing load at once);
//   2. the requests' source runs are put in flight into the warp's shared
//      memory (16-byte cp.async);
//   3. lane (request i, quad c) runs the short filter of channels 4c .. 4c+3
//      (verify_gate4), x2 and u to shared memory;
//   4. each lane advances its channel's 16 modes position by position in
//      packed f32x2 arithmetic (two modes per instruction, the same roundings):
//      each snapshot is written over the channel's modes in the run and the
//      warp stores the run with 16-byte stores, so the padding columns travel
//      from the source block, except channel 0's (the stamp), which are never
//      written; the readout (modal_readout16_x2), D and the x2 gate follow.
// Same arithmetic, order and rounding as decode_kernel.
constexpr int LW_R = 4;        // requests per warp: 8 gate items each fill the warp
constexpr int LW_WARPS = 4;    // warps (32-channel groups) per block

struct LwMeta {
  float u[LW_R][VQ][32], x2[LW_R][VQ][32];
  long long src[LW_R], cin[LW_R], cout[LW_R], dst[LW_R][VQ];
  int t0[LW_R], n[LW_R], off[LW_R], flags[LW_R];
};
static_assert(sizeof(LwMeta) % 16 == 0, "runs follow the metadata 16-byte aligned");
// dynamic shared memory per warp: the metadata, then LW_R runs of 32 D floats
__host__ __device__ constexpr int lw_warp_bytes(int D) { return (int)sizeof(LwMeta) + LW_R * 32 * D * 4; }

__global__ void __launch_bounds__(LW_WARPS * 32)
decode_iir_verify_kernel(const hyena_layer_params P, const hyena_decode_args A) {
  extern __shared__ __align__(16) uint8_t lw_sm[];
  constexpr int F_ZERO = 1, F_SRC = 2, F_CONV = 4;  // flags; snapshot p written: bit 8 + p
  pdl_entry();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int D = (int)A.inner_state.dim_stride;
  LwMeta& M = *reinterpret_cast<LwMeta*>(lw_sm + warp * lw_warp_bytes(D));
  float* runs = reinterpret_cast<float*>(lw_sm + warp * lw_warp_bytes(D) + sizeof(LwMeta));
  const int h0 = (blockIdx.x * LW_WARPS + warp) * 32;  // the warp's first channel
  if (h0 >= P.H) return;  // whole warps only: no block-wide barrier follows
  const int r0 = blockIdx.y * LW_R;
  const long long bs = A.inner_state.block_stride;
  float* st = static_cast<float*>(A.inner_state.data);

  // 1. routing
  if (lane < LW_R) {
    const int i = lane, r = r0 + i;
    int t0 = 0, n = 0, off = 0, fl = 0;
    long long cin = -1, cout = -1, src = -1;
    long long ins[VQ], outs[VQ];
#pragma unroll
    for (int p = 0; p < VQ; ++p) ins[p] = outs[p] = -1;
    if (r < A.num_reqs) {
      // the slot tables' q <= VQ columns are read whole, the accepted one
      // picked afterwards
      t0 = r;
      int t1 = r + 1;
      if (A.token_start) {
        t0 = __ldg(A.token_start + r);
        t1 = __ldg(A.token_start + r + 1);
      }
      int acc = A.accepted ? __ldg(A.accepted + r) : 1;
      cin = __ldg(A.conv_in_block + (long long)r * A.conv_in_stride);
      cout = __ldg(A.conv_out_block + (long long)r * A.conv_out_stride);
#pragma unroll
      for (int p = 0; p < VQ; ++p) {
        if (p < A.q) {
          ins[p] = __ldg(A.in_slots + (long long)r * A.in_stride0 + (long long)p * A.in_stride1);
          outs[p] = __ldg(A.out_slots + (long long)r * A.out_stride0 + (long long)p * A.out_stride1);
        }
      }
      n = t1 - t0;
      if (n > A.q || n > VQ) {
        flag_error(A.error_flags, HYENA_FLAG_SEGMENT);
        n = min(A.q, VQ);
      }
      n = max(n, 0);
      acc = max(1, acc);
      if (acc > A.q) {  // past the slot table's columns
        if (n > 0) flag_error(A.error_flags, HYENA_FLAG_SEGMENT);
        acc = A.q;
      }
      off = acc - 1;
#pragma unroll
      for (int p = 0; p < VQ; ++p)
        if (p == off) src = ins[p];
    }
    if (n > 0) {
      const bool cin_ok = block_ok(cin, A.conv_state);
      if ((A.zero_null_rows && cin == A.null_block) || !cin_ok) fl |= F_ZERO;
      if (block_ok(src, A.inner_state)) fl |= F_SRC;
      if (block_ok(cout, A.conv_state) && !(A.skip_null_writes && cout == A.null_block))
        fl |= F_CONV;
      if (!cin_ok || (!(fl & F_ZERO) && !(fl & F_SRC)))
        flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
    }
#pragma unroll
    for (int p = 0; p < VQ; ++p) {
      const long long d = p < n ? outs[p] : -1;
      if (p < n && !(fl & F_ZERO) && block_ok(d, A.inner_state) &&
          !(A.skip_null_writes && d == A.null_block))
        fl |= 256 << p;
      M.dst[i][p] = d;
    }
    M.t0[i] = t0;
    M.n[i] = n;
    M.off[i] = off;
    M.flags[i] = fl;
    M.cin[i] = cin;
    M.cout[i] = cout;
    M.src[i] = src;
  }
  __syncwarp();

  // 2. source runs: 8 D chunks of 16 bytes per request
  const int chunks = 8 * D;
#pragma unroll 1
  for (int i = 0; i < LW_R; ++i) {
    const int fl = M.flags[i];
    if (M.n[i] == 0 || (fl & F_ZERO)) continue;  // uniform
    float* run = runs + i * 32 * D;
    const float* sp = st + M.src[i] * bs + (long long)h0 * D;
    for (int c = lane; c < chunks; c += 32) {
      if (fl & F_SRC)
        cp_async16(run + 4 * c, sp + 4 * c);
      else
        *reinterpret_cast<float4*>(run + 4 * c) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  cp_async_commit();

  // 3. short filter + gate: lane = (request i, channels 4 c .. 4 c + 3)
  {
    const int i = lane >> 3, c = lane & 7;
    if (M.n[i] > 0 && !(M.flags[i] & F_ZERO)) {
      float x2v[VQ][4], uv[VQ][4];
      verify_gate4<VQ>(P, A, h0 + 4 * c, M.t0[i], M.n[i], M.off[i], M.cin[i], M.cout[i],
                       (M.flags[i] & F_CONV) != 0, x2v, uv);
#pragma unroll
      for (int p = 0; p < VQ; ++p)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          M.x2[i][p][4 * c + k] = x2v[p][k];
          M.u[i][p][4 * c + k] = uv[p][k];
        }
    }
  }
  const int h = h0 + lane;
  float2 pl2[8], rs2[8];
  {
    const float4* lp4 = reinterpret_cast<const float4*>(P.log_poles + (long long)h * P.lp_stride_h);
    const float4* rs4 = reinterpret_cast<const float4*>(P.residues + (long long)h * P.res_stride_h);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 a = __ldg(lp4 + k), b = __ldg(rs4 + k);
      pl2[2 * k] = make_float2(expf(a.x), expf(a.y));
      pl2[2 * k + 1] = make_float2(expf(a.z), expf(a.w));
      rs2[2 * k] = make_float2(b.x, b.y);
      rs2[2 * k + 1] = make_float2(b.z, b.w);
    }
  }
  const bf16* Dg = static_cast<const bf16*>(P.D);
  const float dval = Dg ? ldbf(Dg + h) : 0.0f;
  cp_async_wait<0>();
  __syncwarp();

  // 4. modal recurrence, snapshots, readout, output gate
  const bool stamp_run = D > 16 && h0 == 0;  // chunk 4 holds channel 0's columns 16 ..
  bf16* outp = static_cast<bf16*>(A.out) + h;
#pragma unroll 1
  for (int i = 0; i < LW_R; ++i) {
    const int n = M.n[i], fl = M.flags[i];
    if (n == 0) continue;  // uniform
    const int t0 = M.t0[i];
    if (fl & F_ZERO) {
      for (int p = 0; p < n; ++p) outp[(long long)(t0 + p) * A.ldo] = __float2bfloat16_rn(0.0f);
      continue;
    }
    float* run = runs + i * 32 * D;
    float* mine = run + lane * D;  // odd D: the lanes' rows hit distinct banks
    float2 s2[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) s2[k] = make_float2(mine[2 * k], mine[2 * k + 1]);
#pragma unroll
    for (int p = 0; p < VQ; ++p) {
      if (p >= n) break;  // uniform
      const float u = M.u[i][p][lane];
      const float2 u2 = make_float2(u, u);
#pragma unroll
      for (int k = 0; k < 8; ++k) s2[k] = fadd2(fmul2(s2[k], pl2[k]), u2);
      if (fl & (256 << p)) {  // uniform
        __syncwarp();  // the previous snapshot's stores have read the run
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          mine[2 * k] = s2[k].x;
          mine[2 * k + 1] = s2[k].y;
        }
        __syncwarp();
        float* dp = st + M.dst[i][p] * bs + (long long)h0 * D;
        for (int j = lane; j < chunks; j += 32) {
          const float4 v = *reinterpret_cast<const float4*>(run + 4 * j);
          if (stamp_run && j == 4) {
            const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (16 + k >= D) dp[16 + k] = e[k];
          } else {
            *reinterpret_cast<float4*>(dp + 4 * j) = v;
          }
        }
      }
      float y = bf16r(modal_readout16_x2(s2, rs2));
      if (Dg) y = bf16r(y + bf16r(dval * u));
      outp[(long long)(t0 + p) * A.ldo] = __float2bfloat16_rn(bf16r(M.x2[i][p][lane] * y));
    }
  }
}

// The LI verify path: gate4_ok, S2 rows of 16 .. 20 contiguous floats in
// 16-byte-aligned blocks, poles / residues rows as 16-byte vectors.
static bool iir_verify_ok(const hyena_layer_params& P, const hyena_decode_args& A) {
  if (P.kind != HYENA_KIND_IIR || P.K != 16 || !gate4_ok(P, A)) return false;
  const hyena_state_view& s = A.inner_state;
  return s.col_stride == 1 && s.dim_stride >= 16 && s.dim_stride <= IIR_STAGE_MAXD &&
         aligned_elems(s.data, s.block_stride, 4, 16) && P.lp_stride_s == 1 &&
         P.res_stride_s == 1 && aligned_elems(P.log_poles, P.lp_stride_h, 4, 16) &&
         aligned_elems(P.residues, P.res_stride_h, 4, 16) && P.H % 32 == 0;
}

int decode_launch(const hyena_layer_params& P, const hyena_decode_args& args, cudaStream_t st) {
  hyena_decode_args A = args;
  if (A.conv_in_stride == 0) A.conv_in_stride = 1;
  if (A.conv_out_stride == 0) A.conv_out_stride = 1;
  if (A.conv_state.cols > DEC_MAXW0)
    return fail(HYENA_ERR_UNSUPPORTED, "conv window wider than 8 columns");
  if (fast_path_ok(P, A)) {
    if (P.kind == HYENA_KIND_IIR && P.K == 16) {
      dim3 g((A.num_reqs + LQ_R - 1) / LQ_R, (P.H + LQ_THREADS - 1) / LQ_THREADS);
      launch_kernel(decode_iir_q1_lane_kernel, dim3(g), dim3(LQ_THREADS), 0, st, 0u, P, A);
      return check_launch("decode_iir_q1_lane_kernel");
    }
    dim3 g(A.num_reqs, (P.H / 4 + Q1_THREADS - 1) / Q1_THREADS);
    if (P.kind == HYENA_KIND_FIR && P.K == 128) {
      launch_kernel(decode_fir_q1_kernel<128>, dim3(g), dim3(Q1_THREADS), 0, st, 0u, P, A);
      return check_launch("decode_fir_q1_kernel<128>");
    }
    if (P.kind == HYENA_KIND_FIR && P.K == 7) {
      launch_kernel(decode_fir_q1_kernel<7>, dim3(g), dim3(Q1_THREADS), 0, st, 0u, P, A);
      return check_launch("decode_fir_q1_kernel<7>");
    }
  }
  if (fir_verify_ok(P, A) && (P.K == 128 || P.K == 7)) {
    dim3 g(A.num_reqs, (P.H / 4 + FAST_THREADS - 1) / FAST_THREADS);
    if (P.K == 128)
      launch_kernel(decode_fir_verify_kernel<128>, dim3(g), dim3(FAST_THREADS), 0, st, 0u, P, A);
    else
      launch_kernel(decode_fir_verify_kernel<7>, dim3(g), dim3(FAST_THREADS), 0, st, 0u, P, A);
    return check_launch("decode_fir_verify_kernel");
  }
  if (iir_verify_ok(P, A)) {
    const int bytes = LW_WARPS * lw_warp_bytes((int)A.inner_state.dim_stride);
    if (!smem_attr<decode_iir_verify_kernel>(LW_WARPS * lw_warp_bytes(IIR_STAGE_MAXD)))
      return fail(HYENA_ERR_CUDA, "cudaFuncSetAttribute(decode_iir_verify_kernel)");
    dim3 g((P.H / 32 + LW_WARPS - 1) / LW_WARPS, (A.num_reqs + LW_R - 1) / LW_R);
    launch_kernel(decode_iir_verify_kernel, dim3(g), dim3(LW_WARPS * 32), (size_t)bytes, st, 0u,
                  P, A);
    return check_launch("decode_iir_verify_kernel");
  }
  dim3 grid(A.num_reqs, (P.H + DEC_THREADS - 1) / DEC_THREADS);
  if (P.kind == HYENA_KIND_IIR) {
    if (P.K != 16) return fail(HYENA_ERR_UNSUPPORTED, "IIR decode supports modal order 16");
    const hyena_state_view& s = A.inner_state;
    const bool v16 = s.col_stride == 1 && s.dim_stride >= 16 && s.dim_stride <= IIR_STAGE_MAXD &&
                     (s.dim_stride & 1) && (s.block_stride & 3) == 0 &&
                     (reinterpret_cast<uintptr_t>(s.data) & 15u) == 0 && P.lp_stride_s == 1 &&
                     P.res_stride_s == 1 && aligned_elems(P.log_poles, P.lp_stride_h, 4, 16) &&
                     aligned_elems(P.residues, P.res_stride_h, 4, 16);
    if (v16)
      launch_kernel(decode_kernel<HYENA_KIND_IIR, 16, true>, dim3(grid), dim3(DEC_THREADS), 0, st, 0u,
                    P, A);
    else
      launch_kernel(decode_kernel<HYENA_KIND_IIR, 16>, dim3(grid), dim3(DEC_THREADS), 0, st, 0u, P, A);
  } else if (P.K == 128) {
    launch_kernel(decode_kernel<HYENA_KIND_FIR, 128>, dim3(grid), dim3(DEC_THREADS), 0, st, 0u, P, A);
  } else if (P.K == 7) {
    launch_kernel(decode_kernel<HYENA_KIND_FIR, 7>, dim3(grid), dim3(DEC_THREADS), 0, st, 0u, P, A);
  } else {
    return fail(HYENA_ERR_UNSUPPORTED, "FIR decode supports K = 7 or 128");
  }
  return check_launch("decode_kernel");
}

}  // namespace hb
