// SwinV2 scaled-cosine window attention (reference: src/cpu.rs:1244-1402,
// tools/network_swin2sr.py:151-190).
//
// Persistent CTAs, each owning a group of HPC heads and walking windows: one producer
// warp and 4*HPC compute warps, one (head, 16-query-row block) task per compute warp
// and window, with no block-wide barrier in the window loop. The group's position-bias
// table ([HPC][64][64] fp32, columns XOR-swizzled by row % 8 for conflict-free reads)
// is brought into shared memory once; the producer gathers each window's q/k/v rows of
// those heads by
// bulk copies into one of two buffers (full/empty mbarriers), so the next window's
// copies overlap this window's math. The QKV projection's epilogue has already
// L2-normalised q and k and scaled q by exp(min(logit_scale, ln 100)) * log2 e, and the
// bias table is stored times log2 e, so per window and head:
//   S = Q K^T          mma.sync m16n8k16 fp16 -> fp32 (16 x 64 per warp, in registers)
//   t = S + cpb[h][q][k]   (- 100 log2 e across shift regions, in the last window row
//       and column only; a token's region comes from its rolled plane coordinate)
//   softmax along the row in registers (quad shuffles), max-subtracted, by exp2
//   O = P V            mma.sync, P re-used from the S accumulators as fp16 A fragments
//   out[token][h*hd + d] = O / rowsum
// The residual stream and every token-row buffer stay in image order; this kernel
// is the only place the window partition and cyclic roll exist: `rows` maps the
// window-major token (b, wi, t) of the block's shift to its image row
// (src/plan.rs:72-78), so the window's q/k/v rows (fp16, [heads][q|k|v][DP] per token,
// pad lanes zero) are gathered with one bulk copy per token row into a padded,
// bank-conflict-free shared-memory layout, and outputs are scattered back to the
// same rows.
//
// SPLIT (two-term operands, the 60-wide network): every QKV row carries a second
// fp16 term lo = fp16(x - hi) `lo_q` halves after the first, gathered beside it;
//   S = Qhi Khi^T + Qlo Khi^T + Qhi Klo^T,   O = P Vhi + P Vlo
// and the output is written as hi and lo terms too (lo `lo_out` halves after hi).
// The dot products then carry about 21 bits of the operands instead of 11.
#include "common.cuh"

namespace s2s {
namespace {

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// DP: padded head dim (16 or 32); HPC heads per CTA; SPLIT: two-term operands.
// Window of 64 tokens (win = 8). row_h: halves per QKV token row.
template <int DP, int HPC, bool SPLIT>
__global__ void __launch_bounds__(128 * HPC + 32, SPLIT ? 3 : (HPC == 1 ? 5 : 1)) k_window_attention(
    const __half* __restrict__ qkv, __half* __restrict__ out, const float* __restrict__ cpb,
    const int* __restrict__ rows, int heads, int hd, int ld_out, int row_h, int lo_q, int lo_out,
    int nwh, int nww, int hp, int wp, int shift, int nwin_total, int wh_off) {
  constexpr int N = 64;
  constexpr int NS = N;                        // bias row (floats), XOR-swizzled by row % 8
  constexpr int SEG = HPC * 3 * DP;            // halves of this CTA's heads per token row
  constexpr int SROW = SPLIT ? 2 * SEG : SEG;  // with the lo terms after the hi terms
  constexpr int SSTRIDE = SROW + 8;            // padded smem row: odd number of 16 B units
  static_assert(((SSTRIDE * 2 / 16) & 1) == 1, "bank-conflict-free row stride");
  constexpr int CW = 4 * HPC;                  // compute warps
  extern __shared__ uint8_t smem_raw[];
  float* scpb = reinterpret_cast<float*>(smem_raw);                       // [HPC][64][NS]
  __half* sqb = reinterpret_cast<__half*>(scpb + HPC * N * NS);           // [2][64][SSTRIDE]
  uint64_t* full = reinterpret_cast<uint64_t*>(sqb + 2 * N * SSTRIDE);    // [2]
  uint64_t* empty = full + 2;                                             // [2]
  uint64_t* cbar = empty + 2;                                             // bias table

  const int NG = heads / HPC;
  const int h0 = (blockIdx.x % NG) * HPC;     // first head of this CTA
  const int wstep = gridDim.x / NG;           // host launches a multiple of NG CTAs
  const int nw = nwh * nww;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int win0 = blockIdx.x / NG;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; b++) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], CW);
    }
    mbar_init(cbar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();
  // the bias table is a weight: it loads while the previous kernel finishes
  if (warp == CW && lane == 0) {
    mbar_arrive_expect_tx(cbar, (uint32_t)(HPC * N * NS * 4));
    bulk_g2s(scpb, cpb + (size_t)h0 * N * NS, HPC * N * NS * 4, cbar);
  }
  pdl_wait();  // QKV is complete

  if (warp == CW) {
    // ------------------------------------------------------------ producer warp
    int i = 0;
    for (int win = win0; win < nwin_total; win += wstep, i++) {
      const int b = i & 1;
      // rows of this window (loaded before waiting, so their latency overlaps the wait)
      const int r0 = rows[(size_t)win * N + lane], r1 = rows[(size_t)win * N + 32 + lane];
      if (i >= 2 && !mbar_wait(&empty[b], ((i >> 1) - 1) & 1, DEV_TIMEOUT_EMPTY)) break;
      if (lane == 0) mbar_arrive_expect_tx(&full[b], (uint32_t)(N * SROW * 2));
      __syncwarp();
      __half* dst = sqb + (size_t)b * N * SSTRIDE;
      const __half* s0 = qkv + (size_t)r0 * row_h + h0 * 3 * DP;
      const __half* s1 = qkv + (size_t)r1 * row_h + h0 * 3 * DP;
      bulk_g2s(dst + (size_t)lane * SSTRIDE, s0, SEG * 2, &full[b]);
      bulk_g2s(dst + (size_t)(32 + lane) * SSTRIDE, s1, SEG * 2, &full[b]);
      if constexpr (SPLIT) {
        bulk_g2s(dst + (size_t)lane * SSTRIDE + SEG, s0 + lo_q, SEG * 2, &full[b]);
        bulk_g2s(dst + (size_t)(32 + lane) * SSTRIDE + SEG, s1 + lo_q, SEG * 2, &full[b]);
      }
    }
    return;
  }

  // -------------------------------------------------------------- compute warps
  const int g = lane >> 2, t4 = lane & 3;
  const int hl = warp >> 2, rb = warp & 3;     // this warp's task in every window
  const int h = h0 + hl;
  const int qr0 = rb * 16 + g, qr1 = qr0 + 8;
  const int qoff = hl * 3 * DP, koff = qoff + DP, voff = qoff + 2 * DP;
  const float* cp0 = scpb + ((size_t)hl * N + qr0) * NS;
  const float* cp1 = scpb + ((size_t)hl * N + qr1) * NS;
  const uint32_t sbase0 = smem_u32(sqb);
  bool ok = mbar_wait(cbar, 0, DEV_TIMEOUT_FULL);
  const int nwh_g = hp / 8;                   // window rows of the rolled plane
  constexpr float kMask = -100.0f * 1.4426950408889634f;  // -100, in the exp2 domain

  int i = 0;
  // this thread's two output rows of the first window (the next window's are loaded
  // while this one computes)
  int orow0 = 0, orow1 = 0;
  if (win0 < nwin_total) {
    orow0 = rows[(size_t)win0 * N + qr0];
    orow1 = rows[(size_t)win0 * N + qr1];
  }
  for (int win = win0; win < nwin_total && ok; win += wstep, i++) {
    const int b = i & 1;
    const int cur0 = orow0, cur1 = orow1;
    if (win + wstep < nwin_total) {
      orow0 = rows[(size_t)(win + wstep) * N + qr0];
      orow1 = rows[(size_t)(win + wstep) * N + qr1];
    }
    if (!mbar_wait(&full[b], (i >> 1) & 1, DEV_TIMEOUT_FULL)) break;
    const uint32_t sbase = sbase0 + (uint32_t)(b * N * SSTRIDE * 2);
    const int wi = win % nw;
    // window row on the (global) hp x wp plane the shift mask is defined on
    int wh = wi / nww + wh_off;
    if (wh < 0) wh += nwh_g;
    const int ww = wi % nww;
    // Only the last window row and column of a shifted block mix roll regions.
    const bool masked = shift && (wh == nwh_g - 1 || ww == nww - 1);
    int qreg0 = 0, qreg1 = 0;
    if (masked) {
      qreg0 = 3 * region_of(wh * 8 + qr0 / 8, hp, 8, shift) + region_of(ww * 8 + qr0 % 8, wp, 8, shift);
      qreg1 = 3 * region_of(wh * 8 + qr1 / 8, hp, 8, shift) + region_of(ww * 8 + qr1 % 8, wp, 8, shift);
    }

    // S = Q K^T for 16 rows x 64 keys.
    float sacc[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < DP / 16; kk++) {
      uint32_t a0, a1, a2, a3, l0 = 0, l1 = 0, l2 = 0, l3 = 0;
      const int arow = rb * 16 + (lane & 15);
      const int acol = qoff + kk * 16 + (lane >> 4) * 8;
      ldsm_x4(sbase + (uint32_t)((arow * SSTRIDE + acol) * 2), a0, a1, a2, a3);
      if constexpr (SPLIT) ldsm_x4(sbase + (uint32_t)((arow * SSTRIDE + acol + SEG) * 2), l0, l1, l2, l3);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int krow = 8 * j + (lane & 7) + ((lane >> 4) << 3);
        const int kcol = koff + kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(sbase + (uint32_t)((krow * SSTRIDE + kcol) * 2), b0, b1, b2, b3);
        mma16816(sacc[j], a0, a1, a2, a3, b0, b1);
        mma16816(sacc[j + 1], a0, a1, a2, a3, b2, b3);
        if constexpr (SPLIT) {
          mma16816(sacc[j], l0, l1, l2, l3, b0, b1);
          mma16816(sacc[j + 1], l0, l1, l2, l3, b2, b3);
          ldsm_x4(sbase + (uint32_t)((krow * SSTRIDE + kcol + SEG) * 2), b0, b1, b2, b3);
          mma16816(sacc[j], a0, a1, a2, a3, b0, b1);
          mma16816(sacc[j + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }

    // Bias, mask, softmax (q and k arrive normalised, q scaled by the clamped logit
    // scale times log2 e; the bias table is pre-scaled by log2 e).
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int k = 8 * j + 2 * t4;
      const int ks = k ^ (g << 2);  // both query rows have row % 8 == g
      const float2 b0 = *reinterpret_cast<const float2*>(cp0 + ks);
      const float2 b1 = *reinterpret_cast<const float2*>(cp1 + ks);
      float s00 = sacc[j][0] + b0.x;
      float s01 = sacc[j][1] + b0.y;
      float s10 = sacc[j][2] + b1.x;
      float s11 = sacc[j][3] + b1.y;
      if (masked) {
        const int kr0 = 3 * region_of(wh * 8 + k / 8, hp, 8, shift) + region_of(ww * 8 + k % 8, wp, 8, shift);
        const int kr1 = 3 * region_of(wh * 8 + (k + 1) / 8, hp, 8, shift) +
                        region_of(ww * 8 + (k + 1) % 8, wp, 8, shift);
        if (qreg0 != kr0) s00 += kMask;
        if (qreg0 != kr1) s01 += kMask;
        if (qreg1 != kr0) s10 += kMask;
        if (qreg1 != kr1) s11 += kMask;
      }
      sacc[j][0] = s00;
      sacc[j][1] = s01;
      sacc[j][2] = s10;
      sacc[j][3] = s11;
      mx0 = fmaxf(mx0, fmaxf(s00, s01));
      mx1 = fmaxf(mx1, fmaxf(s10, s11));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      sacc[j][0] = ex2(sacc[j][0] - mx0);
      sacc[j][1] = ex2(sacc[j][1] - mx0);
      sacc[j][2] = ex2(sacc[j][2] - mx1);
      sacc[j][3] = ex2(sacc[j][3] - mx1);
      sum0 += sacc[j][0] + sacc[j][1];
      sum1 += sacc[j][2] + sacc[j][3];
    }
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);

    // O = P V.
    float oacc[DP / 8][4];
#pragma unroll
    for (int n = 0; n < DP / 8; n++) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      const uint32_t a0 = pack_h2(sacc[2 * kk][0], sacc[2 * kk][1]);
      const uint32_t a1 = pack_h2(sacc[2 * kk][2], sacc[2 * kk][3]);
      const uint32_t a2 = pack_h2(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
      const uint32_t a3 = pack_h2(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
#pragma unroll
      for (int n = 0; n < DP / 8; n += 2) {
        uint32_t b0, b1, b2, b3;
        const int vrow = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int vcol = voff + n * 8 + ((lane >> 4) << 3);
        ldsm_x4_t(sbase + (uint32_t)((vrow * SSTRIDE + vcol) * 2), b0, b1, b2, b3);
        mma16816(oacc[n], a0, a1, a2, a3, b0, b1);
        mma16816(oacc[n + 1], a0, a1, a2, a3, b2, b3);
        if constexpr (SPLIT) {
          ldsm_x4_t(sbase + (uint32_t)((vrow * SSTRIDE + vcol + SEG) * 2), b0, b1, b2, b3);
          mma16816(oacc[n], a0, a1, a2, a3, b0, b1);
          mma16816(oacc[n + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    // this warp is done with the buffer
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[b]);
    const float inv0 = 1.0f / sum0, inv1 = 1.0f / sum1;
    __half* o0 = out + (size_t)cur0 * ld_out + h * hd;
    __half* o1 = out + (size_t)cur1 * ld_out + h * hd;
#pragma unroll
    for (int n = 0; n < DP / 8; n++) {
      const int d = n * 8 + 2 * t4;
      if (d < hd) {
        const float v00 = oacc[n][0] * inv0, v01 = oacc[n][1] * inv0;
        const float v10 = oacc[n][2] * inv1, v11 = oacc[n][3] * inv1;
        const __half2 h0 = __floats2half2_rn(v00, v01), h1 = __floats2half2_rn(v10, v11);
        *reinterpret_cast<__half2*>(o0 + d) = h0;
        *reinterpret_cast<__half2*>(o1 + d) = h1;
        if constexpr (SPLIT) {
          const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
          *reinterpret_cast<__half2*>(o0 + lo_out + d) = __floats2half2_rn(v00 - f0.x, v01 - f0.y);
          *reinterpret_cast<__half2*>(o1 + lo_out + d) = __floats2half2_rn(v10 - f1.x, v11 - f1.y);
        }
      }
    }
  }
}

template <int DP, bool SPLIT>
cudaError_t launch_attn_t(const __half* qkv, __half* out, const float* cpb, const int* rows,
                          int nwin_total, int heads, int hd, int ld_out, int row_h, int lo_q,
                          int lo_out, int nwh, int nww, int hp, int wp, int shift, int wh_off,
                          cudaStream_t st) {
  constexpr int HPC = 1;
  constexpr int SEG = HPC * 3 * DP, SROW = SPLIT ? 2 * SEG : SEG;
  const size_t smem = (size_t)HPC * 64 * 64 * 4 + (size_t)2 * 64 * (SROW + 8) * 2 + 5 * 8 + 16;
  static LaunchSetup setup;  // resident CTAs, per device
  int ctas = 0;
  const cudaError_t err =
      resident_ctas(setup, k_window_attention<DP, HPC, SPLIT>, 128 * HPC + 32, smem, &ctas);
  if (err != cudaSuccess) return err;
  const int NG = heads / HPC;
  long G = (long)nwin_total * NG;
  if (G > ctas) G = ctas;
  G = (G / NG) * NG;
  if (G < NG) G = NG;
  return launch_pdl(k_window_attention<DP, HPC, SPLIT>, dim3((unsigned)G), dim3(128 * HPC + 32),
                    smem, st, qkv, out, cpb, rows, heads, hd, ld_out, row_h, lo_q, lo_out, nwh,
                    nww, hp, wp, shift, nwin_total, wh_off);
}

}  // namespace

// One head per CTA: the smallest CTA (about 43 KB of shared memory), so five fit on an
// SM and their window streams hide each other's latency (two heads per CTA, two CTAs
// per SM, measured 11 % slower). row_h: halves per QKV token row; split: the rows
// carry lo terms lo_q halves after the hi terms, and the output gets its lo terms
// lo_out halves after hi.
cudaError_t launch_window_attention(const __half* qkv, __half* out, const float* cpb,
                                    const int* rows, int nwin_total, int heads, int hd, int dp,
                                    int ld_out, int row_h, int split, int lo_q, int lo_out,
                                    int nwh, int nww, int hp, int wp, int shift, int wh_off,
                                    cudaStream_t st) {
  if (row_h < 3 * heads * dp || (split && (lo_q < 3 * heads * dp || row_h < lo_q + 3 * heads * dp)))
    return cudaErrorInvalidValue;
  if (dp == 32 && !split)
    return launch_attn_t<32, false>(qkv, out, cpb, rows, nwin_total, heads, hd, ld_out, row_h, 0,
                                    0, nwh, nww, hp, wp, shift, wh_off, st);
  if (dp == 32)
    return launch_attn_t<32, true>(qkv, out, cpb, rows, nwin_total, heads, hd, ld_out, row_h, lo_q,
                                   lo_out, nwh, nww, hp, wp, shift, wh_off, st);
  if (dp == 16 && !split)
    return launch_attn_t<16, false>(qkv, out, cpb, rows, nwin_total, heads, hd, ld_out, row_h, 0,
                                    0, nwh, nww, hp, wp, shift, wh_off, st);
  if (dp == 16)
    return launch_attn_t<16, true>(qkv, out, cpb, rows, nwin_total, heads, hd, ld_out, row_h, lo_q,
                                   lo_out, nwh, nww, hp, wp, shift, wh_off, st);
  return cudaErrorInvalidValue;
}

}  // namespace s2s
