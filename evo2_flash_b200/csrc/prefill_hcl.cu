// Hyena-LI (HCL) prefill for sm_100a: the order-16 diagonal modal SSM
//     s_t = p (.) s_{t-1} + u_t,   y_t = sum_s R_s s_{t,s},   p = exp(log_poles)
// over packed varlen segments, fused with the K=3 short filter, the x1*v gate
// and the (y + D*u) * x2 output gate.
//
// The reference computes the same map as an FFT convolution with the
// materialised modal filter h[l] = sum_s R_s p_s^l plus a closed-form final
// state and the s_prev continuation terms (mixers.py:144-210, 1378-1397;
// triton_hcl.py:88-123; triton_prefill.py:351-387).  Here it is a chunked
// Toeplitz contraction on the tensor cores.  Per channel, a 512-row tile is a
// 16 x 32 matrix U(j, tau) = u[t0 + 32 j + tau] (row j = one 32-row chunk) and
//   A    = U . G          G(tau, s) = p_s^(31-tau)     chunk aggregates (16 x 16)
//   S_in = carry over the 16 chunks (S_in(j+1) = p^32 (.) S_in(j) + A(j)), a
//          Kogge-Stone scan across the lanes that hold the rows of A
//   Y    = U . T + S_in . V
//          T(tau, i) = h[i - tau] (i >= tau)  the intra-chunk Toeplitz filter
//          V(s, i)   = R_s p_s^(i+1)          the carried state's readout
// with every operand in bf16 for mma.sync m16n8k16 (fp32 accumulation): u is
// bf16 already, and the fp32 operands (h, p powers, S_in) are split into
// hi + lo bf16 pairs (about 16 significant bits), so the products carry fp32-
// level accuracy.  The aggregate's C fragment is, lane for lane, the A-operand
// layout of the S_in . V product, so the carried states never leave registers.
// A segment's final state is the recurrence over its last partial chunk from
// that chunk's S_in (one thread per mode).
//
// Work split: a CTA owns 8 channels (one warp each in the tensor phase) and a
// range of one segment's rows, which it walks tile by tile, carrying the modal
// state: z is read from HBM once.  Segments longer than the range length R
// (chosen so that the grid fills the GPU) are split into ranges; then a first
// pass computes every non-final range's end state from zero (aggregates only),
// a carry kernel chains them per (segment, channel, mode), and the main pass
// starts each range from its carried state.  Every launch is order-independent
// across CTAs: no inter-CTA waits.
#include "common.cuh"

namespace hb {

constexpr int HCL_CG = 8;        // channels per CTA (one warp per channel)
constexpr int HCL_PAIRS = HCL_CG / 2;
constexpr int HCL_THREADS = 256;
constexpr int HCL_BT = 512;      // rows per tile
constexpr int HCL_C = 32;        // rows per chunk
constexpr int HCL_NJ = HCL_BT / HCL_C;
constexpr int HCL_S = 16;        // modal order
constexpr int HCL_RPT = 8;       // rows per thread in the gate and store phases
constexpr int HCL_WORDS = 3 * HCL_PAIRS;                              // z words per row
constexpr int HCL_ZT_WORDS = HCL_WORDS * HCL_BT + 4 * (HCL_BT / 8);   // one z tile
constexpr int HCL_CH = (HCL_BT / 32) * 5 + 1;  // 16-byte chunks per channel (odd stride)
constexpr int HCL_STAGES = 3;
constexpr int HCL_TARGET_CTAS = 148 * 8;

static_assert(HCL_PAIRS * (HCL_BT / HCL_RPT) == HCL_THREADS, "gate mapping");
static_assert(HCL_THREADS / 32 == HCL_CG, "one warp per channel");

struct HclPlan {
  int32_t* range_base;  // (nseg + 1): ranges before segment j
  float* states;        // (max_ranges, H, 16): range aggregates, then start states
  int R;                // rows per range (multiple of HCL_BT)
};

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Rows per range: a multiple of the tile, large enough that the (groups x
// ranges) grid is about HCL_TARGET_CTAS, so short segments stay whole.
static int hcl_range_rows(int H, int T) {
  const long long groups = H / HCL_CG;
  long long r = ((long long)T * groups + HCL_TARGET_CTAS - 1) / HCL_TARGET_CTAS;
  r = (r + HCL_BT - 1) / HCL_BT * HCL_BT;
  return (int)(r < HCL_BT ? HCL_BT : (r > (1 << 30) ? (1 << 30) : r));
}
static int hcl_max_ranges(int H, int T, int nseg) {
  const int R = hcl_range_rows(H, T);
  return (T + R - 1) / R + nseg;
}

size_t hcl_workspace_size(int H, int T, int nseg) {
  return align_up(sizeof(int32_t) * (size_t)(nseg + 1), 256) +
         sizeof(float) * (size_t)hcl_max_ranges(H, T, nseg) * (size_t)H * HCL_S;
}

static HclPlan carve(void* ws, int nseg, int R) {
  HclPlan w;
  w.range_base = static_cast<int32_t*>(ws);
  w.states = reinterpret_cast<float*>(static_cast<char*>(ws) +
                                      align_up(sizeof(int32_t) * (size_t)(nseg + 1), 256));
  w.R = R;
  return w;
}

// Segment rows clamped to the T rows of z / out.
__device__ __forceinline__ int seg_row(const int32_t* qsl, int j, int T) {
  return max(0, min(__ldg(qsl + j), T));
}

__global__ void hcl_plan_kernel(const int32_t* qsl, int nseg, int T, int R, int32_t* range_base) {
  pdl_entry();
  if (threadIdx.x != 0) return;
  int acc = 0;
  for (int j = 0; j < nseg; ++j) {
    range_base[j] = acc;
    const int L = seg_row(qsl, j + 1, T) - seg_row(qsl, j, T);
    acc += L > 0 ? (L + R - 1) / R : 0;
  }
  range_base[nseg] = acc;
}

struct RangeCtx {
  int seg, k, nch;  // segment, range within segment, ranges of the segment
  int a, e;         // segment rows
  int row0, row1;   // range rows
  long long blk;
  bool init;
};

// Returns false when range ci does not exist.
__device__ __forceinline__ bool range_ctx(const hyena_prefill_args& A, const HclPlan& W, int ci,
                                          RangeCtx& c) {
  const int nseg = A.num_segments;
  const int32_t* rb = W.range_base;
  if (ci >= __ldg(rb + nseg)) return false;
  // last j with rb[j] <= ci: segments without ranges share their base with the
  // next one, so this is the owning (non-empty) segment
  const int j = find_segment(rb, nseg, ci);
  c.seg = j;
  c.k = ci - __ldg(rb + j);
  c.nch = __ldg(rb + j + 1) - __ldg(rb + j);
  c.a = seg_row(A.query_start_loc, j, A.T);
  c.e = seg_row(A.query_start_loc, j + 1, A.T);
  c.row0 = c.a + c.k * W.R;
  c.row1 = min(c.e, c.row0 + W.R);
  c.blk = __ldg(A.state_indices + (long long)j * A.state_indices_stride);
  c.init = A.has_initial_state != nullptr && __ldg(A.has_initial_state + j) != 0;
  return true;
}

struct HclShared {
  uint32_t zt[HCL_STAGES][HCL_ZT_WORDS];  // z tiles, bf16x2 words
  uint4 ub[HCL_CG * HCL_CH];               // u by (channel, tile row), bf16
  uint4 ys[HCL_CG * HCL_CH];               // y by (channel, tile row), bf16
  // (p_s^32)^e, e = 0..16; a stride of 20 per mode keeps the scan's lanes
  // (mode 2q + c, power g) on 32 different banks
  float pw[HCL_CG][HCL_S][20];
  float pole[HCL_CG][HCL_S];               // p_s
  float hf[HCL_CG][HCL_C];                 // modal filter h[l], l < 32
  float sfin[HCL_CG][HCL_S];               // S_in of a segment's last chunk
  uint32_t zh[2][2][HCL_WORDS];            // z rows (r-2, r-1) before the tile, [tile parity]
  bf162 sw[3][3][HCL_PAIRS];               // short taps [column][tap][pair]
  bf162 dsm[HCL_PAIRS];
};

// Word offset of z tile row r (a 4-word gap after every 8 rows).
__device__ __forceinline__ int hzrow(int r) { return r * HCL_WORDS + 4 * (r >> 3); }
// 16-byte chunk of (channel, rows 8c .. 8c+7) in ub / ys: per channel, lines of
// 32 rows (one chunk of the tensor phase's U / Y) at an 80-byte pitch, which
// keeps every ldmatrix / stmatrix phase and the gate and store phases free of
// bank conflicts.
__device__ __forceinline__ int hchunk(int ch, int c) { return ch * HCL_CH + 5 * (c >> 2) + (c & 3); }

__device__ __forceinline__ uint32_t hsmem(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void hldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(hsmem(p))
               : "memory");
}
__device__ __forceinline__ void hstsm_x4(void* p, uint32_t r0, uint32_t r1, uint32_t r2,
                                         uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(hsmem(p)),
               "r"(r0), "r"(r1), "r"(r2), "r"(r3)
               : "memory");
}
// d += a . b, m16n8k16, bf16 operands, fp32 accumulators.
__device__ __forceinline__ void hmma(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ uint32_t hpack(float lo, float hi) {
  return as_u32(__floats2bfloat162_rn(lo, hi));
}
// x = hi + mid + lo, each bf16, |x - hi - mid - lo| <= 2^-24 |x| (each
// remainder is exact in fp32): bf16x2 words of two values.
__device__ __forceinline__ void hsplit3(float x0, float x1, uint32_t& hi, uint32_t& mid,
                                        uint32_t& lo) {
  const bf162 h = __floats2bfloat162_rn(x0, x1);
  const float2 hf = __bfloat1622float2(h);
  const float r0 = x0 - hf.x, r1 = x1 - hf.y;
  const bf162 m = __floats2bfloat162_rn(r0, r1);
  const float2 mf = __bfloat1622float2(m);
  hi = as_u32(h);
  mid = as_u32(m);
  lo = hpack(r0 - mf.x, r1 - mf.y);
}

__device__ __forceinline__ uint32_t hbits(float v) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// z at row t (absolute column col) with the segment's left context: rows
// before the segment come from the cached S0 window, or are zero.
__device__ __forceinline__ float hz_at(const hyena_prefill_args& A, const RangeCtx& c, long long t,
                                       int col) {
  if (t >= c.a) return ldbf(static_cast<const bf16*>(A.z) + t * A.ldz + col);
  if (!c.init) return 0.0f;
  const long long back = c.a - t;  // 1 = newest cached input, in column 1
  if (back > 2) return 0.0f;
  const bf16* s0 = static_cast<const bf16*>(A.conv_state.data);
  return ldbf(s0 + c.blk * A.conv_state.block_stride + (2 - back) * A.conv_state.col_stride +
              (long long)col * A.conv_state.dim_stride);
}

// The interleaved triple words of one channel pair, w0 = (x2_a, x1_a),
// w1 = (v_a, x2_b), w2 = (x1_b, v_b) -> bf16x2 pairs of one column.
__device__ __forceinline__ bf162 hsplit_x2(uint32_t w0, uint32_t w1) {
  return as_bf162(__byte_perm(w0, w1, 0x7610));
}
__device__ __forceinline__ void hsplit_x1v(uint32_t w0, uint32_t w1, uint32_t w2, bf162& x1,
                                           bf162& v) {
  x1 = as_bf162(__byte_perm(w0, w2, 0x5432));
  v = as_bf162(__byte_perm(w1, w2, 0x7610));
}

// Issues the z rows [r, r + n) of this CTA's channels into buffer buf and
// closes one cp.async group (empty when n == 0).  Thread (group gi, row rin,
// chunk v) copies rows 8 gi + rin + 80 k: row offsets in the gapped tile then
// advance by a constant.
__device__ __forceinline__ void hcl_prefetch(HclShared& S, const hyena_prefill_args& A, int r0,
                                             int n, int buf, int c0) {
  constexpr int VPR = HCL_WORDS * 4 / 16;                      // 16-byte chunks per row
  constexpr int PASS = (HCL_THREADS / (8 * VPR)) * 8;          // rows per pass
  constexpr int DST_STEP = PASS * HCL_WORDS + 4 * (PASS / 8);  // hzrow(r + PASS) - hzrow(r)
  const int tid = threadIdx.x;
  if (tid < PASS * VPR) {
    const int v = tid % VPR;
    int r = 8 * (tid / (8 * VPR)) + (tid % (8 * VPR)) / VPR;
    uint32_t* dst = &S.zt[buf][hzrow(r) + 4 * v];
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const bf16*>(A.z) +
                                                      (long long)(r0 + r) * A.ldz + 3 * c0) + v;
    const long long step = (long long)PASS * A.ldz / 8;  // in 16-byte units
    for (; r < n; r += PASS, dst += DST_STEP, src += step) cp_async16(dst, src);
  }
  cp_async_commit();
}

// One CTA: channels [8 blockIdx.x, +8) of range blockIdx.y.  AGG: aggregates
// only (the range's end state from a zero start, into W.states); otherwise
// the full output, starting from the range's carried state.
template <bool AGG>
__global__ void __launch_bounds__(HCL_THREADS, 2)
hcl_tc_kernel(const hyena_layer_params P, const hyena_prefill_args A, HclPlan W) {
  pdl_entry();
  extern __shared__ __align__(16) unsigned char hcl_smem_raw[];
  HclShared& S = *reinterpret_cast<HclShared*>(hcl_smem_raw);
  RangeCtx c;
  if (!range_ctx(A, W, blockIdx.y, c)) return;
  if (AGG && c.k == c.nch - 1) return;  // the final range's end state is the segment's own
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = blockIdx.x * HCL_CG;
  const bool blk_ok = c.blk >= 0 && c.blk < A.inner_state.num_blocks &&
                      c.blk < A.conv_state.num_blocks;
  if (c.init && !blk_ok) c.init = false;

  // ---- first z tiles in flight
  const int nrows = c.row1 - c.row0;
  const int ntiles = (nrows + HCL_BT - 1) / HCL_BT;
  hcl_prefetch(S, A, c.row0, min(HCL_BT, nrows), 0, c0);
#pragma unroll
  for (int s = 1; s < HCL_STAGES - 1; ++s) {
    const int r = c.row0 + s * HCL_BT;
    hcl_prefetch(S, A, r, max(0, min(HCL_BT, c.row1 - r)), s, c0);
  }

  // ---- parameters: poles, powers, the modal filter, short taps, D, z history
  const float* lpg = P.log_poles;
  const float* rsg = P.residues;
  for (int i = tid; i < HCL_CG * HCL_S; i += HCL_THREADS) {
    const int ch = i / HCL_S, s = i % HCL_S;
    const float lp = lpg[(long long)(c0 + ch) * P.lp_stride_h + (long long)s * P.lp_stride_s];
    S.pole[ch][s] = expf(lp);
#pragma unroll
    for (int e = 0; e <= HCL_NJ; ++e) S.pw[ch][s][e] = expf(lp * (float)(HCL_C * e));
  }
  {
    const int ch = tid / HCL_C, l = tid % HCL_C;  // 8 x 32 = 256 threads
    float acc = 0.0f;
#pragma unroll
    for (int s = 0; s < HCL_S; ++s) {
      const long long h = c0 + ch;
      acc = fmaf(rsg[h * P.res_stride_h + (long long)s * P.res_stride_s],
                 expf(lpg[h * P.lp_stride_h + (long long)s * P.lp_stride_s] * (float)l), acc);
    }
    S.hf[ch][l] = acc;
  }
  {
    const bf16* swg = static_cast<const bf16*>(P.short_w);
    for (int i = tid; i < 9 * HCL_PAIRS; i += HCL_THREADS) {
      const int col = i / (3 * HCL_PAIRS), tap = (i / HCL_PAIRS) % 3, pp = i % HCL_PAIRS;
      const long long h = c0 + 2 * pp;
      S.sw[col][tap][pp] = __halves2bfloat162(swg[(3 * h + col) * 3 + tap],
                                              swg[(3 * (h + 1) + col) * 3 + tap]);
    }
    const bf16* Dg = static_cast<const bf16*>(P.D);
    if (tid < HCL_PAIRS)
      S.dsm[tid] = Dg ? __halves2bfloat162(Dg[c0 + 2 * tid], Dg[c0 + 2 * tid + 1])
                      : __floats2bfloat162_rn(0.f, 0.f);
    for (int i = tid; i < 2 * HCL_WORDS; i += HCL_THREADS) {
      const int q = i / HCL_WORDS, wd = i % HCL_WORDS;
      const long long t = (long long)c.row0 - 2 + q;
      S.zh[0][q][wd] = hbits(hz_at(A, c, t, 3 * c0 + 2 * wd)) |
                    (hbits(hz_at(A, c, t, 3 * c0 + 2 * wd + 1)) << 16);
    }
  }
  __syncthreads();

  // ---- constant B fragments of this warp's channel (k16 x n8: b0 = (k = 2q, 2q+1; n = g),
  // b1 = (k + 8; n = g)), each split into hi / mid / lo bf16 so that the products
  // with the bf16 data carry fp32 accuracy
  const int ch = warp, g = lane >> 2, q = lane & 3;
  const int h = c0 + ch;
  const float* lph = lpg + (long long)h * P.lp_stride_h;
  uint32_t G3[3][2][2][2];  // [split][ks][n-tile][b]: G(tau = 16 ks + 8 b + 2q (+1), s = 8 n + g)
#pragma unroll
  for (int ks = 0; ks < 2; ++ks)
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const int tau = 16 * ks + 8 * b + 2 * q;
        const float lp = lph[(long long)(8 * n + g) * P.lp_stride_s];
        hsplit3(expf(lp * (float)(HCL_C - 1 - tau)), expf(lp * (float)(HCL_C - 2 - tau)),
                G3[0][ks][n][b], G3[1][ks][n][b], G3[2][ks][n][b]);
      }
  uint32_t V3[3][4][2];  // [split][n-tile][b]: V(s = 8 b + 2q (+1), i = 8 n + g) = R_s p_s^(i+1)
  {
    const float* rr = rsg + (long long)h * P.res_stride_h;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const int s = 8 * b + 2 * q, i = 8 * n + g;
        const float v0 = rr[(long long)s * P.res_stride_s] *
                         expf(lph[(long long)s * P.lp_stride_s] * (float)(i + 1));
        const float v1 = rr[(long long)(s + 1) * P.res_stride_s] *
                         expf(lph[(long long)(s + 1) * P.lp_stride_s] * (float)(i + 1));
        hsplit3(v0, v1, V3[0][n][b], V3[1][n][b], V3[2][n][b]);
      }
  }
  // T(tau, i) = h[i - tau] (i >= tau) depends on i - tau only: the fragment of
  // (k-step ks, n-tile n) has b0 = word(8 n - 16 ks), b1 = word(8 n - 16 ks - 8)
  // with word(x) = (h[x + g - 2q], h[x + g - 2q - 1]); five words cover the
  // nonzero blocks (ks 0 x n 0..3, ks 1 x n 2..3): x = -8, 0, 8, 16, 24.
  uint32_t T3[3][5];
#pragma unroll
  for (int w = 0; w < 5; ++w) {
    const int i0 = 8 * w - 8 + g - 2 * q;
    const float t0 = i0 >= 0 ? S.hf[ch][i0] : 0.0f;
    const float t1 = i0 - 1 >= 0 ? S.hf[ch][i0 - 1] : 0.0f;
    hsplit3(t0, t1, T3[0][w], T3[1][w], T3[2][w]);
  }

  // ---- carried modal state: this lane's modes 2q, 2q+1, 8+2q, 9+2q
  float carry[4];
  const float* st2 = static_cast<const float*>(A.inner_state.data);
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const int s = 8 * (m >> 1) + 2 * q + (m & 1);
    if (AGG) {
      carry[m] = 0.0f;
    } else if (c.nch > 1) {
      carry[m] = W.states[((long long)blockIdx.y * P.H + h) * HCL_S + s];
    } else {
      carry[m] = c.init ? st2[c.blk * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride +
                              (long long)s * A.inner_state.col_stride]
                        : 0.0f;
    }
  }

  // gate / store mapping: an 8-lane phase holds 4 channel pairs x 2 row groups
  const int pp = lane & 3;
  const int rg = warp * 8 + (lane >> 2);
  const int g0 = rg * HCL_RPT;
  bf16* out = static_cast<bf16*>(A.out);
  const bool has_d = P.D != nullptr;
  int buf = 0;
  int zc = 0;  // the zh buffer holding the current tile's z history

  for (int it = 0; it < ntiles; ++it) {
    const int r = c.row0 + it * HCL_BT;
    const int n = min(HCL_BT, c.row1 - r);
    __syncthreads();  // the previous tile is finished (z buffer, ub, ys, zh)
    {
      const int rn = r + (HCL_STAGES - 1) * HCL_BT;
      hcl_prefetch(S, A, rn, max(0, min(HCL_BT, c.row1 - rn)), (buf + HCL_STAGES - 1) % HCL_STAGES,
                   c0);
    }
    cp_async_wait<HCL_STAGES - 1>();
    __syncthreads();
    const uint32_t* zt = S.zt[buf];

    // rows g0 - 2, g0 - 1 of this thread's channel pair (z history at g0 = 0)
    const uint32_t* zga = g0 >= 2 ? &zt[hzrow(g0 - 2) + 3 * pp] : &S.zh[zc][g0][3 * pp];
    const uint32_t* zgb = g0 >= 1 ? &zt[hzrow(g0 - 1) + 3 * pp] : &S.zh[zc][1][3 * pp];
    const uint32_t* zg = &zt[hzrow(g0) + 3 * pp];  // rows g0.. of one 8-row group
    // ---- gate phase: K=3 short filter of the x1 and v columns on a channel pair
    // over 8 consecutive rows, u = x1 * v (x2 is filtered in the store phase)
    if (g0 < n) {
      bf162 w[2][3];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc)
#pragma unroll
        for (int k = 0; k < 3; ++k) w[cc][k] = S.sw[cc + 1][k][pp];
      bf162 h2[2], h1[2];
      hsplit_x1v(zga[0], zga[1], zga[2], h2[0], h2[1]);
      hsplit_x1v(zgb[0], zgb[1], zgb[2], h1[0], h1[1]);
      uint32_t uu[HCL_RPT];
#pragma unroll
      for (int i = 0; i < HCL_RPT; ++i) {
        const uint32_t* zr = zg + i * HCL_WORDS;
        bf162 cur[2], o[2];
        hsplit_x1v(zr[0], zr[1], zr[2], cur[0], cur[1]);
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          o[cc] = short_tap2(h2[cc], h1[cc], cur[cc], w[cc][0], w[cc][1], w[cc][2]);
          h2[cc] = h1[cc];
          h1[cc] = cur[cc];
        }
        // rows past the range read stale shared memory: their u must be zero
        uu[i] = g0 + i < n ? as_u32(__hmul2(o[0], o[1])) : 0u;
      }
      uint4 ua, ubv;
      ua.x = __byte_perm(uu[0], uu[1], 0x5410); ubv.x = __byte_perm(uu[0], uu[1], 0x7632);
      ua.y = __byte_perm(uu[2], uu[3], 0x5410); ubv.y = __byte_perm(uu[2], uu[3], 0x7632);
      ua.z = __byte_perm(uu[4], uu[5], 0x5410); ubv.z = __byte_perm(uu[4], uu[5], 0x7632);
      ua.w = __byte_perm(uu[6], uu[7], 0x5410); ubv.w = __byte_perm(uu[6], uu[7], 0x7632);
      S.ub[hchunk(2 * pp, rg)] = ua;
      S.ub[hchunk(2 * pp + 1, rg)] = ubv;
    } else {
      const uint4 zero = make_uint4(0, 0, 0, 0);  // rows past the range: u = 0
      S.ub[hchunk(2 * pp, rg)] = zero;
      S.ub[hchunk(2 * pp + 1, rg)] = zero;
    }
    __syncthreads();

    // ---- tensor phase (warp = channel)
    {
      // U fragments: A operand (16 chunks x 32 rows); matrix mi = (row half, k half)
      uint32_t Ua[2][4];
      {
        const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks)
          hldsm_x4(Ua[ks], &S.ub[ch * HCL_CH + 5 * (rr + 8 * (mi & 1)) + (mi >> 1) + 2 * ks]);
      }
      // chunk aggregates A (16 chunks x 16 modes)
      float accA[2][4];
#pragma unroll
      for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int e = 0; e < 4; ++e) accA[nn][e] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
#pragma unroll
        for (int nn = 0; nn < 2; ++nn)
#pragma unroll
          for (int sp = 2; sp >= 0; --sp) hmma(accA[nn], Ua[ks], G3[sp][ks][nn]);
      // carry over the chunks: inclusive Kogge-Stone scan of each row half over
      // the lanes g (stride 4), halves joined, then S_in(j) = P^j carry + E(j-1)
      float sin_lo[4], sin_hi[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float* pws = &S.pw[ch][8 * (m >> 1) + 2 * q + (m & 1)][0];
        float elo = accA[m >> 1][m & 1], ehi = accA[m >> 1][2 + (m & 1)];
#pragma unroll
        for (int d = 1; d < 8; d *= 2) {
          const float ulo = __shfl_up_sync(0xffffffffu, elo, 4 * d);
          const float uhi = __shfl_up_sync(0xffffffffu, ehi, 4 * d);
          if (g >= d) {
            elo = fmaf(pws[d], ulo, elo);
            ehi = fmaf(pws[d], uhi, ehi);
          }
        }
        const float e7 = __shfl_sync(0xffffffffu, elo, 28 + q);
        ehi = fmaf(pws[g + 1], e7, ehi);
        const float plo = __shfl_up_sync(0xffffffffu, elo, 4);
        const float phi = __shfl_up_sync(0xffffffffu, ehi, 4);
        const float e15 = __shfl_sync(0xffffffffu, ehi, 28 + q);
        sin_lo[m] = fmaf(pws[g], carry[m], g >= 1 ? plo : 0.0f);
        sin_hi[m] = fmaf(pws[g + 8], carry[m], g >= 1 ? phi : e7);
        carry[m] = fmaf(pws[HCL_NJ], carry[m], e15);
      }
      if (!AGG) {
        // S_in as the A operand (16 chunks x 16 modes), hi / mid / lo
        uint32_t S3[3][4];
        hsplit3(sin_lo[0], sin_lo[1], S3[0][0], S3[1][0], S3[2][0]);
        hsplit3(sin_hi[0], sin_hi[1], S3[0][1], S3[1][1], S3[2][1]);
        hsplit3(sin_lo[2], sin_lo[3], S3[0][2], S3[1][2], S3[2][2]);
        hsplit3(sin_hi[2], sin_hi[3], S3[0][3], S3[1][3], S3[2][3]);
        float accY[4][4];
#pragma unroll
        for (int nn = 0; nn < 4; ++nn)
#pragma unroll
          for (int e = 0; e < 4; ++e) accY[nn][e] = 0.0f;
        // smaller terms first: the carried-state readout (every product of
        // order >= 2^-16 of the leading one), then the intra-chunk Toeplitz
#pragma unroll
        for (int nn = 0; nn < 4; ++nn) {
          hmma(accY[nn], S3[1], V3[1][nn]);
          hmma(accY[nn], S3[2], V3[0][nn]);
          hmma(accY[nn], S3[0], V3[2][nn]);
          hmma(accY[nn], S3[1], V3[0][nn]);
          hmma(accY[nn], S3[0], V3[1][nn]);
          hmma(accY[nn], S3[0], V3[0][nn]);
        }
#pragma unroll
        for (int f = 0; f < 6; ++f) {
          const int ks = f < 4 ? 0 : 1, nn = f < 4 ? f : f - 2;
          const int w0 = nn - 2 * ks + 1;  // word index of x = 8 nn - 16 ks
#pragma unroll
          for (int sp = 2; sp >= 0; --sp) {
            const uint32_t tb[2] = {T3[sp][w0], T3[sp][w0 - 1]};
            hmma(accY[nn], Ua[ks], tb);
          }
        }
        // y (bf16) into the y tile: matrix k = (row half k & 1, n-tile 2x + (k >> 1))
        const int sk = lane >> 3, srr = lane & 7;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const int nn = 2 * x + (sk >> 1);
          hstsm_x4(&S.ys[ch * HCL_CH + 5 * (srr + 8 * (sk & 1)) + nn],
                   hpack(accY[2 * x][0], accY[2 * x][1]), hpack(accY[2 * x][2], accY[2 * x][3]),
                   hpack(accY[2 * x + 1][0], accY[2 * x + 1][1]),
                   hpack(accY[2 * x + 1][2], accY[2 * x + 1][3]));
        }
        // the segment's final state: the recurrence over its last chunk from S_in
        if (r + n == c.e) {
          const int jl = (n - 1) / HCL_C;
          if (g == (jl & 7)) {
#pragma unroll
            for (int m = 0; m < 4; ++m)
              S.sfin[ch][8 * (m >> 1) + 2 * q + (m & 1)] = jl >= 8 ? sin_hi[m] : sin_lo[m];
          }
          __syncwarp();
          if (lane < HCL_S && blk_ok) {
            const int s = lane;
            const float p = S.pole[ch][s];
            float sv = S.sfin[ch][s];
            const bf16* uch = reinterpret_cast<const bf16*>(&S.ub[0]);
            const int last = (n - 1) % HCL_C;
            for (int tau = 0; tau <= last; ++tau) {
              const int row = HCL_C * jl + tau;
              const float uv =
                  __bfloat162float(uch[hchunk(ch, row >> 3) * 8 + (row & 7)]);
              sv = add_rn(mul_rn(sv, p), uv);
            }
            float* st = static_cast<float*>(A.inner_state.data);
            st[c.blk * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride +
               (long long)s * A.inner_state.col_stride] = sv;
          }
          if (lane == 0 && !blk_ok) flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
        }
      }
    }

    if (!AGG) {
      __syncthreads();
      // ---- store phase: g = bf16(x2 * bf16(y + bf16(D * u))) on channel pairs
      if (g0 < n) {
        const uint4 ya = S.ys[hchunk(2 * pp, rg)], yb = S.ys[hchunk(2 * pp + 1, rg)];
        const uint4 ua = S.ub[hchunk(2 * pp, rg)], ubv = S.ub[hchunk(2 * pp + 1, rg)];
        const uint32_t yaw[4] = {ya.x, ya.y, ya.z, ya.w}, ybw[4] = {yb.x, yb.y, yb.z, yb.w};
        const uint32_t uaw[4] = {ua.x, ua.y, ua.z, ua.w}, ubw[4] = {ubv.x, ubv.y, ubv.z, ubv.w};
        const bf162 d2 = S.dsm[pp];
        const bf162 wx0 = S.sw[0][0][pp], wx1 = S.sw[0][1][pp], wx2 = S.sw[0][2][pp];
        bf162 x2h2 = hsplit_x2(zga[0], zga[1]), x2h1 = hsplit_x2(zgb[0], zgb[1]);
        bf162* outp = reinterpret_cast<bf162*>(out + (long long)(r + g0) * A.ldo + c0) + pp;
        const long long ld2 = A.ldo / 2;
#pragma unroll
        for (int i = 0; i < HCL_RPT; ++i) {
          const bf162 x2c = hsplit_x2(zg[i * HCL_WORDS], zg[i * HCL_WORDS + 1]);
          const bf162 x2 = short_tap2(x2h2, x2h1, x2c, wx0, wx1, wx2);
          x2h2 = x2h1;
          x2h1 = x2c;
          if (g0 + i < n) {
            const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
            bf162 y = as_bf162(__byte_perm(yaw[i >> 1], ybw[i >> 1], sel));
            // D*u is rounded to bf16 before the add, as torch does: the _rn
            // multiply keeps the compiler from fusing the two into one bf16 FMA
            if (has_d)
              y = __hadd2(y, __hmul2_rn(d2, as_bf162(__byte_perm(uaw[i >> 1], ubw[i >> 1], sel))));
            outp[i * ld2] = __hmul2(x2, y);
          }
        }
      }
    }
    // ---- z history for the next tile, into the other zh buffer (the store
    // phase may still read this tile's)
    if (tid < HCL_WORDS && n == HCL_BT) {
      S.zh[zc ^ 1][0][tid] = zt[hzrow(HCL_BT - 2) + tid];
      S.zh[zc ^ 1][1][tid] = zt[hzrow(HCL_BT - 1) + tid];
    }
    zc ^= 1;
    buf = (buf + 1) % HCL_STAGES;
  }
  cp_async_wait<0>();

  if (AGG) {  // the range's end state from a zero start (the range is whole tiles)
    if (g == 7) {
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int s = 8 * (m >> 1) + 2 * q + (m & 1);
        W.states[((long long)blockIdx.y * P.H + h) * HCL_S + s] = carry[m];
      }
    }
  }
}

// One thread per (segment, channel, mode) of a segment split into ranges:
// every range's start state, written over that range's end state from zero.
__global__ void __launch_bounds__(128)
hcl_carry_kernel(const hyena_layer_params P, const hyena_prefill_args A, HclPlan W) {
  pdl_entry();
  const int j = blockIdx.x;
  const long long idx = (long long)blockIdx.y * 128 + threadIdx.x;  // h * 16 + s
  if (idx >= (long long)P.H * HCL_S) return;
  const int h = (int)(idx / HCL_S), s = (int)(idx % HCL_S);
  const int base = __ldg(W.range_base + j);
  const int nch = __ldg(W.range_base + j + 1) - base;
  if (nch <= 1) return;  // a whole segment starts from the cached state directly
  const long long blk = __ldg(A.state_indices + (long long)j * A.state_indices_stride);
  bool init = A.has_initial_state != nullptr && __ldg(A.has_initial_state + j) != 0;
  if (init && (blk < 0 || blk >= A.inner_state.num_blocks)) {
    flag_error(A.error_flags, HYENA_FLAG_BLOCK_RANGE);
    init = false;
  }
  const float* s2 = static_cast<const float*>(A.inner_state.data);
  float Sv = init ? s2[blk * A.inner_state.block_stride + (long long)h * A.inner_state.dim_stride +
                       (long long)s * A.inner_state.col_stride]
                  : 0.0f;
  const float pr =
      expf(P.log_poles[(long long)h * P.lp_stride_h + s * P.lp_stride_s] * (float)W.R);
  float* slot = W.states + (long long)base * P.H * HCL_S + idx;
  const long long stride = (long long)P.H * HCL_S;
  for (int k = 0; k < nch; ++k) {
    const float a = k < nch - 1 ? slot[k * stride] : 0.0f;  // read before the overwrite
    slot[k * stride] = Sv;
    Sv = add_rn(mul_rn(pr, Sv), a);
  }
}

int conv_state_update_launch(const hyena_layer_params& P, const hyena_prefill_args& A,
                             cudaStream_t st);

int hcl_prefill_launch(const hyena_layer_params& P, const hyena_prefill_args& A, void* ws,
                       size_t ws_bytes, cudaStream_t st) {
  if (P.K != HCL_S) return fail(HYENA_ERR_UNSUPPORTED, "HCL prefill supports modal order 16");
  if (P.H % HCL_CG) return fail(HYENA_ERR_INVALID, "HCL prefill needs H % 8 == 0");
  const size_t need = hcl_workspace_size(P.H, A.T, A.num_segments);
  if (ws == nullptr || ws_bytes < need)
    return fail(HYENA_ERR_INVALID, "HCL prefill workspace too small");
  if (!aligned16(ws)) return fail(HYENA_ERR_INVALID, "HCL workspace must be 16-byte aligned");
  const int R = hcl_range_rows(P.H, A.T);
  HclPlan W = carve(ws, A.num_segments, R);
  const int max_ranges = hcl_max_ranges(P.H, A.T, A.num_segments);
  const int groups = P.H / HCL_CG;
  launch_kernel(hcl_plan_kernel, dim3(1), dim3(32), 0, st, 0u, A.query_start_loc, A.num_segments,
                A.T, R, W.range_base);
  int rc = check_launch("hcl_plan_kernel");
  if (rc) return rc;
  const int smem = (int)sizeof(HclShared);
  if (!smem_attr<hcl_tc_kernel<true>>(smem) || !smem_attr<hcl_tc_kernel<false>>(smem))
    return fail(HYENA_ERR_CUDA, "cudaFuncSetAttribute(hcl) failed");
  // segments no longer than R (every one, when T <= R) need neither the
  // aggregate pass nor the carry: their CTAs return at once
  if (A.T > R) {
    launch_kernel(hcl_tc_kernel<true>, dim3(groups, max_ranges), dim3(HCL_THREADS), (size_t)smem,
                  st, 0u, P, A, W);
    if ((rc = check_launch("hcl_tc_kernel<aggregate>"))) return rc;
    launch_kernel(hcl_carry_kernel, dim3(A.num_segments, (P.H * HCL_S + 127) / 128), dim3(128), 0,
                  st, 0u, P, A, W);
    if ((rc = check_launch("hcl_carry_kernel"))) return rc;
  }
  launch_kernel(hcl_tc_kernel<false>, dim3(groups, max_ranges), dim3(HCL_THREADS), (size_t)smem,
                st, 0u, P, A, W);
  if ((rc = check_launch("hcl_tc_kernel"))) return rc;
  return conv_state_update_launch(P, A, st);
}

}  // namespace hb
