// SwinV2 scaled-cosine window attention (reference: src/cpu.rs:1244-1402,
// tools/network_swin2sr.py:151-190).
//
// One CTA per 8x8 window, eight warps. The reciprocal L2 norms of every q and k
// row of every head are computed once per window; then each warp takes (head,
// 16-query-row block) tasks independently. Per task:
//   S = Q K^T          mma.sync m16n8k16 fp16 -> fp32 (16 x 64 per warp, in registers)
//   s = S * (1/|q|) * (1/|k|) * exp(min(logit_scale, ln 100)) + cpb[h][q][k]  (- 100 across shift
//       regions; the region of a token is computed from its rolled plane coordinate)
//   softmax along the row in registers (quad shuffles), max-subtracted
//   O = P V            mma.sync, P re-used from the S accumulators as fp16 A fragments
//   out[token][h*hd + d] = O / rowsum
// The residual stream and every token-row buffer stay in image order; this kernel
// is the only place the window partition and cyclic roll exist: `rows` maps the
// window-major token (b, wi, t) of the block's shift to its image row
// (src/plan.rs:72-78), so the window's q/k/v rows (fp16, [3][heads][DP] per token,
// pad lanes zero) are gathered with one bulk copy per token row into a padded,
// bank-conflict-free shared-memory layout, and outputs are scattered back to the
// same rows.
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

__device__ __forceinline__ int region_of(int a, int p, int win, int shift) {
  return (a + win < p) ? 0 : (a + shift < p) ? 1 : 2;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// DP: padded head dim (16 or 32). Window of 64 tokens (win = 8).
template <int DP>
__global__ void __launch_bounds__(256) k_window_attention(
    const __half* __restrict__ qkv, __half* __restrict__ out, const float* __restrict__ cpb,
    const float* __restrict__ lscale, const int* __restrict__ rows, int heads, int hd, int ld_out,
    int nwh, int nww, int hp, int wp, int shift) {
  constexpr int N = 64;
  const int row_h = 3 * heads * DP;            // halves per token row
  const int row_bytes = row_h * 2;
  const int sstride = row_h + 8;               // padded smem row (halves): odd number of 16 B
  extern __shared__ uint8_t smem_raw[];
  __half* sq = reinterpret_cast<__half*>(smem_raw);
  // [heads][2][64]: 1/|k| then 1/|q| per head
  float* snorm = reinterpret_cast<float*>(smem_raw + (size_t)N * sstride * 2);
  uint64_t* bar = reinterpret_cast<uint64_t*>(snorm + 2 * N * heads);

  const int win_idx = blockIdx.x;              // global window (image-major)
  const int nw = nwh * nww;
  const int wi = win_idx % nw;
  const int wh = wi / nww, ww = wi % nww;
  const size_t tok0 = (size_t)win_idx * N;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) mbar_arrive_expect_tx(bar, (uint32_t)(N * row_bytes));
  __syncthreads();
  if (tid < N)
    bulk_g2s(sq + (size_t)tid * sstride, qkv + (size_t)rows[tok0 + tid] * row_h, row_bytes, bar);
  const bool ok = mbar_wait(bar, 0, DEV_TIMEOUT_FULL);
  if (!__syncthreads_and(ok)) return;  // uniform exit: no thread is left at a barrier

  // Reciprocal norms of every head's q and k rows, from the same fp16 values the MMAs read.
  for (int idx = tid; idx < 2 * N * heads; idx += blockDim.x) {
    const int h = idx / (2 * N), rem = idx - h * 2 * N;
    const int isq = rem >= N, tok = rem & (N - 1);
    const __half* v = sq + (size_t)tok * sstride + (isq ? h : heads + h) * DP;
    float acc = 0.0f;
    for (int d = 0; d < hd; d++) {
      const float x = __half2float(v[d]);
      acc += x * x;
    }
    snorm[idx] = 1.0f / fmaxf(sqrtf(acc), 1e-12f);
  }
  __syncthreads();

  const uint32_t sbase = smem_u32(sq);
  for (int task = warp; task < heads * 4; task += 8) {
    const int h = task >> 2, rb = task & 3;
    const int qr0 = rb * 16 + g, qr1 = qr0 + 8;
    int qreg0 = 0, qreg1 = 0;
    if (shift) {
      qreg0 = 3 * region_of(wh * 8 + qr0 / 8, hp, 8, shift) + region_of(ww * 8 + qr0 % 8, wp, 8, shift);
      qreg1 = 3 * region_of(wh * 8 + qr1 / 8, hp, 8, shift) + region_of(ww * 8 + qr1 % 8, wp, 8, shift);
    }
    const int qoff = h * DP, koff = (heads + h) * DP, voff = (2 * heads + h) * DP;

    // S = Q K^T for 16 rows x 64 keys.
    float sacc[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < DP / 16; kk++) {
      uint32_t a0, a1, a2, a3;
      const int arow = rb * 16 + (lane & 15);
      const int acol = qoff + kk * 16 + (lane >> 4) * 8;
      ldsm_x4(sbase + (uint32_t)((arow * sstride + acol) * 2), a0, a1, a2, a3);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int krow = 8 * j + (lane & 7) + ((lane >> 4) << 3);
        const int kcol = koff + kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(sbase + (uint32_t)((krow * sstride + kcol) * 2), b0, b1, b2, b3);
        mma16816(sacc[j], a0, a1, a2, a3, b0, b1);
        mma16816(sacc[j + 1], a0, a1, a2, a3, b2, b3);
      }
    }

    // Scale, bias, mask, softmax.
    const float ls = lscale[h];
    const float* kinv = snorm + h * 2 * N;
    const float qs0 = kinv[N + qr0] * ls, qs1 = kinv[N + qr1] * ls;
    const float* cp0 = cpb + ((size_t)h * N + qr0) * N;
    const float* cp1 = cpb + ((size_t)h * N + qr1) * N;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int k = 8 * j + 2 * t4;
      const float ki0 = kinv[k], ki1 = kinv[k + 1];
      const float2 b0 = __ldg(reinterpret_cast<const float2*>(cp0 + k));
      const float2 b1 = __ldg(reinterpret_cast<const float2*>(cp1 + k));
      float s00 = sacc[j][0] * ki0 * qs0 + b0.x;
      float s01 = sacc[j][1] * ki1 * qs0 + b0.y;
      float s10 = sacc[j][2] * ki0 * qs1 + b1.x;
      float s11 = sacc[j][3] * ki1 * qs1 + b1.y;
      if (shift) {
        const int kr0 = 3 * region_of(wh * 8 + k / 8, hp, 8, shift) + region_of(ww * 8 + k % 8, wp, 8, shift);
        const int kr1 = 3 * region_of(wh * 8 + (k + 1) / 8, hp, 8, shift) +
                        region_of(ww * 8 + (k + 1) % 8, wp, 8, shift);
        if (qreg0 != kr0) s00 -= 100.0f;
        if (qreg0 != kr1) s01 -= 100.0f;
        if (qreg1 != kr0) s10 -= 100.0f;
        if (qreg1 != kr1) s11 -= 100.0f;
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
      sacc[j][0] = __expf(sacc[j][0] - mx0);
      sacc[j][1] = __expf(sacc[j][1] - mx0);
      sacc[j][2] = __expf(sacc[j][2] - mx1);
      sacc[j][3] = __expf(sacc[j][3] - mx1);
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
        ldsm_x4_t(sbase + (uint32_t)((vrow * sstride + vcol) * 2), b0, b1, b2, b3);
        mma16816(oacc[n], a0, a1, a2, a3, b0, b1);
        mma16816(oacc[n + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    const float inv0 = 1.0f / sum0, inv1 = 1.0f / sum1;
    __half* o0 = out + (size_t)rows[tok0 + qr0] * ld_out + h * hd;
    __half* o1 = out + (size_t)rows[tok0 + qr1] * ld_out + h * hd;
#pragma unroll
    for (int n = 0; n < DP / 8; n++) {
      const int d = n * 8 + 2 * t4;
      if (d < hd) {
        *reinterpret_cast<__half2*>(o0 + d) =
            __floats2half2_rn(oacc[n][0] * inv0, oacc[n][1] * inv0);
        *reinterpret_cast<__half2*>(o1 + d) =
            __floats2half2_rn(oacc[n][2] * inv1, oacc[n][3] * inv1);
      }
    }
  }
}

}  // namespace

cudaError_t launch_window_attention(const __half* qkv, __half* out, const float* cpb,
                                    const float* lscale, const int* rows, int nwin_total,
                                    int heads, int hd, int dp, int ld_out, int nwh, int nww,
                                    int hp, int wp, int shift, cudaStream_t st) {
  const int row_h = 3 * heads * dp;
  const size_t smem = (size_t)64 * (row_h + 8) * 2 + 2 * 64 * heads * 4 + 16;
  if (dp == 32) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(k_window_attention<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      set = true;
    }
    k_window_attention<32><<<nwin_total, 256, smem, st>>>(qkv, out, cpb, lscale, rows, heads, hd,
                                                          ld_out, nwh, nww, hp, wp, shift);
  } else if (dp == 16) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(k_window_attention<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      set = true;
    }
    k_window_attention<16><<<nwin_total, 256, smem, st>>>(qkv, out, cpb, lscale, rows, heads, hd,
                                                          ld_out, nwh, nww, hp, wp, shift);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace s2s
