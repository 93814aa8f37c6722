// The HBM-bound pieces around the tensor-core kernels: reflect padding of the
// input plane, the 3-input-channel convolutions (conv_first, conv_after_aux,
// conv_bicubic), the bicubic resample of the compressed head, and the nearest
// x2 upsample of the real-world head.
#include <algorithm>

#include "common.cuh"

namespace s2s {
namespace {

// src/plan.rs:116-139: [B][c][h][w] -> [B][c][hp][wp], whole-plane mirror.
__global__ void k_pad_reflect(const float* __restrict__ x, float* __restrict__ y, int B, int c,
                              int h, int w, int hp, int wp) {
  pdl_trigger();
  pdl_wait();
  const size_t n = (size_t)B * c * hp * wp;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int xx = (int)(i % wp);
    const int yy = (int)((i / wp) % hp);
    const size_t bc = i / ((size_t)wp * hp);
    const int sy = yy < h ? yy : 2 * h - 1 - min(yy, 2 * h - 1);
    const int sx = xx < w ? xx : 2 * w - 1 - min(xx, 2 * w - 1);
    y[i] = x[(bc * h + sy) * w + sx];
  }
}

// One row band of the padded plane: rows [y0, y0 + rows) of the hp x wp mirror of
// k_pad_reflect, zero outside [0, hp) (the 3x3 convolution's padding at the plane's
// true edges).
__global__ void k_pad_band(const float* __restrict__ x, float* __restrict__ y, int c, int h,
                           int w, int hp, int wp, int rows, int y0) {
  pdl_trigger();
  pdl_wait();
  const size_t n = (size_t)c * rows * wp;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int xx = (int)(i % wp);
    const int ly = (int)((i / wp) % rows);
    const int ch = (int)(i / ((size_t)wp * rows));
    const int yy = y0 + ly;
    float v = 0.0f;
    if (yy >= 0 && yy < hp) {
      const int sy = yy < h ? yy : 2 * h - 1 - min(yy, 2 * h - 1);
      const int sx = xx < w ? xx : 2 * w - 1 - min(xx, 2 * w - 1);
      v = x[((size_t)ch * h + sy) * w + sx];
    }
    y[i] = v;
  }
}

// 3x3 s1 p1 conv with 3 input channels, NCHW fp32 input -> NHWC outputs.
// A warp is 32 consecutive pixels of one row and one group of 8 output channels:
// the input loads coalesce across the warp, the weights are shared-memory
// broadcasts (two channels' weights per float2, feeding one packed f32x2 fma), and
// each thread stores its pixel's 8 channels as 32 + 16 bytes.
// Taps in the oracle's order: bias first, then ky, kx, ci.
constexpr int kConvGroups = 8;  // channel groups per block (blockDim = 32 x 8)
__global__ void __launch_bounds__(256) k_conv3_small(
    const float* __restrict__ in, const float* __restrict__ wgt, const float* __restrict__ bias,
    int B, int H, int W, int co_n, int act, float slope, float* __restrict__ o32, int ld32,
    __half* __restrict__ o16, int ld16, int lo16) {
  // weights of output channels (2p, 2p + 1) side by side: one float2 per tap feeds a
  // packed two-channel fma
  __shared__ float2 sw2[kConvGroups * 4][27];
  __shared__ float sb[kConvGroups * 8];
  const int lane = threadIdx.x, g = threadIdx.y;
  const int cbase = blockIdx.y * kConvGroups * 8;
  for (int i = g * 32 + lane; i < kConvGroups * 8 * 27; i += 256) {
    const int cl = i / 27, co = cbase + cl;
    const float wv = co < co_n ? wgt[(size_t)co * 27 + i % 27] : 0.0f;
    if (cl & 1)
      sw2[cl >> 1][i % 27].y = wv;
    else
      sw2[cl >> 1][i % 27].x = wv;
  }
  for (int i = g * 32 + lane; i < kConvGroups * 8; i += 256)
    sb[i] = cbase + i < co_n ? bias[cbase + i] : 0.0f;
  pdl_trigger();
  pdl_wait();  // the input plane is complete
  __syncthreads();
  const int c0 = cbase + g * 8;  // this warp's first output channel
  if (c0 >= co_n) return;
  const int tiles_x = (W + 31) / 32;
  const size_t ntiles = (size_t)B * H * tiles_x;
  for (size_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int tx = (int)(t % tiles_x);
    const int y = (int)((t / tiles_x) % H);
    const int b = (int)(t / ((size_t)tiles_x * H));
    const int x = tx * 32 + lane;
    if (x >= W) continue;
    float v[27];
#pragma unroll
    for (int ci = 0; ci < 3; ci++)
#pragma unroll
      for (int ky = 0; ky < 3; ky++)
#pragma unroll
        for (int kx = 0; kx < 3; kx++) {
          const int sy = y + ky - 1, sx = x + kx - 1;
          v[ci * 9 + ky * 3 + kx] = (sy >= 0 && sy < H && sx >= 0 && sx < W)
                                        ? in[(((size_t)b * 3 + ci) * H + sy) * W + sx]
                                        : 0.0f;
        }
    unsigned long long v2[27];  // each input twice: one operand for two channels
#pragma unroll
    for (int t = 0; t < 27; t++) v2[t] = f2_pack(v[t], v[t]);
    float acc[8];
#pragma unroll
    for (int jp = 0; jp < 4; jp++) {
      // channels 2jp, 2jp+1 of this warp: bias first, then ky, kx, ci, one fma each
      const float2* wc = sw2[g * 4 + jp];
      unsigned long long a2 = f2_pack(sb[g * 8 + 2 * jp], sb[g * 8 + 2 * jp + 1]);
#pragma unroll
      for (int ky = 0; ky < 3; ky++)
#pragma unroll
        for (int kx = 0; kx < 3; kx++)
#pragma unroll
          for (int ci = 0; ci < 3; ci++) {
            const int t = ci * 9 + ky * 3 + kx;
            const float2 w2 = wc[t];
            a2 = f2_fma(f2_pack(w2.x, w2.y), v2[t], a2);
          }
      const float2 a = f2_unpack(a2);
      acc[2 * jp] = (act == 2 && a.x < 0.0f) ? a.x * slope : a.x;
      acc[2 * jp + 1] = (act == 2 && a.y < 0.0f) ? a.y * slope : a.y;
    }
    const size_t p = ((size_t)b * H + y) * W + x;
    const int nv = min(8, co_n - c0);
    if (nv == 8) {
      if (o32) {
        float4* d = reinterpret_cast<float4*>(o32 + p * ld32 + c0);
        d[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        d[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      }
      if (o16) {
        uint4 u;
        __half2 h0 = __floats2half2_rn(acc[0], acc[1]), h1 = __floats2half2_rn(acc[2], acc[3]);
        __half2 h2 = __floats2half2_rn(acc[4], acc[5]), h3 = __floats2half2_rn(acc[6], acc[7]);
        u.x = *reinterpret_cast<uint32_t*>(&h0);
        u.y = *reinterpret_cast<uint32_t*>(&h1);
        u.z = *reinterpret_cast<uint32_t*>(&h2);
        u.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(o16 + p * ld16 + c0) = u;
        if (lo16) {  // two-term operand: the remainder of each fp16 value, at lo16
          const __half2 hs[4] = {h0, h1, h2, h3};
          uint32_t lw[4];
#pragma unroll
          for (int m = 0; m < 4; m++) {
            const float2 f = __half22float2(hs[m]);
            const __half2 l = __floats2half2_rn(acc[2 * m] - f.x, acc[2 * m + 1] - f.y);
            lw[m] = *reinterpret_cast<const uint32_t*>(&l);
          }
          *reinterpret_cast<uint4*>(o16 + p * ld16 + lo16 + c0) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j < nv) {
          if (o32) o32[p * ld32 + c0 + j] = acc[j];
          if (o16) {
            const __half hv = __float2half_rn(acc[j]);
            o16[p * ld16 + c0 + j] = hv;
            if (lo16) o16[p * ld16 + lo16 + c0 + j] = __float2half_rn(acc[j] - __half2float(hv));
          }
        }
    }
  }
}

// Zero the pad channels [c0, ld) of NHWC rows (so padded K lanes are finite zeros).
__global__ void k_zero_cols_f16(__half* __restrict__ x, size_t rows, int c0, int ld) {
  pdl_trigger();
  pdl_wait();
  const int w = ld - c0;
  const size_t n = rows * w;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    x[(i / w) * ld + c0 + (i % w)] = __float2half_rn(0.0f);
}

// src/cpu.rs:877-935: torch bicubic, a = -0.75, align_corners = False, edge clamp.
__device__ __forceinline__ float cubic_w(float t) {
  const float A = -0.75f;
  t = fabsf(t);
  if (t <= 1.0f) return ((A + 2.0f) * t - (A + 3.0f)) * t * t + 1.0f;
  if (t < 2.0f) return (((t - 5.0f) * t + 8.0f) * t - 4.0f) * A;
  return 0.0f;
}

__global__ void k_bicubic(const float* __restrict__ in, float* __restrict__ out, int BC, int h,
                          int w, int oh, int ow) {
  pdl_trigger();
  pdl_wait();
  const size_t n = (size_t)BC * oh * ow;
  const float ry = (float)h / (float)oh, rx = (float)w / (float)ow;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int x = (int)(i % ow);
    const int y = (int)((i / ow) % oh);
    const size_t bc = i / ((size_t)ow * oh);
    const float sy = ((float)y + 0.5f) * ry - 0.5f, sx = ((float)x + 0.5f) * rx - 0.5f;
    const float by = floorf(sy), bx = floorf(sx);
    int iy[4], ix[4];
    float wy[4], wx[4];
#pragma unroll
    for (int m = 0; m < 4; m++) {
      iy[m] = min(max((int)by - 1 + m, 0), h - 1);
      ix[m] = min(max((int)bx - 1 + m, 0), w - 1);
      wy[m] = cubic_w(sy - (by + (float)m - 1.0f));
      wx[m] = cubic_w(sx - (bx + (float)m - 1.0f));
    }
    const float* src = in + bc * h * w;
    float acc = 0.0f;
#pragma unroll
    for (int m = 0; m < 4; m++) {
      const float* r = src + (size_t)iy[m] * w;
      const float a0 = wx[0] * r[ix[0]], a1 = wx[1] * r[ix[1]];
      const float a2 = wx[2] * r[ix[2]], a3 = wx[3] * r[ix[3]];
      acc += wy[m] * ((a0 + a1) + (a2 + a3));
    }
    out[i] = acc;
  }
}

// Nearest x2 upsample of an NHWC fp16 plane, 16 bytes per thread.
__global__ void k_up2_nhwc(const __half* __restrict__ in, __half* __restrict__ out, int B, int H,
                           int W, int C) {
  pdl_trigger();
  pdl_wait();
  const int cv = C / 8;
  const size_t n = (size_t)B * 2 * H * 2 * W * cv;
  const uint4* src = reinterpret_cast<const uint4*>(in);
  uint4* dst = reinterpret_cast<uint4*>(out);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % cv);
    const size_t p = i / cv;
    const int x = (int)(p % (2 * W));
    const int y = (int)((p / (2 * W)) % (2 * H));
    const int b = (int)(p / ((size_t)4 * W * H));
    dst[i] = src[(((size_t)b * H + (y >> 1)) * W + (x >> 1)) * cv + c];
  }
}

// The continuous position bias of one block, computed once on the device from the
// checkpoint's MLP (network_swin2sr.py:103-137; the table tools/convert.py:141-167
// precomputes): for query q and key k of a win x win window, relative entry
// e = (dy + win - 1) * (2 win - 1) + (dx + win - 1) of the log-spaced coordinate table,
//   cpb[h][q][k] = 16 * sigmoid( sum_j w2[h][j] * relu(w0[j] . t_e + b0[j]) ).
// Stored as the attention kernel reads it: times log2 e, key column k at
// k ^ ((q % 8) * 4). Thread per (head, query, key).
__global__ void k_cpb_table(const float* __restrict__ table, const float* __restrict__ w0,
                            const float* __restrict__ b0, const float* __restrict__ w2, int heads,
                            int win, int hidden, float* __restrict__ out) {
  const int n = win * win;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= heads * n * n) return;
  const int h = i / (n * n), q = (i / n) % n, k = i % n;
  const int e = (q / win - k / win + win - 1) * (2 * win - 1) + (q % win - k % win + win - 1);
  const float t0 = table[2 * e], t1 = table[2 * e + 1];
  const float* wh = w2 + (size_t)h * hidden;
  float acc = 0.0f;
  for (int j = 0; j < hidden; j++) {
    const float z = t0 * w0[2 * j] + t1 * w0[2 * j + 1] + b0[j];
    acc += fmaxf(z, 0.0f) * wh[j];
  }
  const float v = 16.0f / (1.0f + expf(-acc));
  out[((size_t)h * n + q) * n + (k ^ ((q & 7) << 2))] = v * 1.4426950408889634f;
}

inline unsigned grid_for(size_t n, int block) {
  size_t g = (n + block - 1) / block;
  if (g > 148 * 64) g = 148 * 64;
  return (unsigned)(g == 0 ? 1 : g);
}

}  // namespace

cudaError_t launch_pad_reflect(const float* x, float* y, int B, int c, int h, int w, int hp,
                               int wp, cudaStream_t st) {
  return launch_pdl(k_pad_reflect, dim3(grid_for((size_t)B * c * hp * wp, 256)), dim3(256), 0, st, x,
                    y, B, c, h, w, hp, wp);
}

cudaError_t launch_pad_band(const float* x, float* y, int c, int h, int w, int hp, int wp, int rows,
                            int y0, cudaStream_t st) {
  return launch_pdl(k_pad_band, dim3(grid_for((size_t)c * rows * wp, 256)), dim3(256), 0, st, x, y,
                    c, h, w, hp, wp, rows, y0);
}

cudaError_t launch_conv3_small(const float* in, const float* wgt, const float* bias, int B, int H,
                               int W, int co_n, int act, float slope, float* o32, int ld32,
                               __half* o16, int ld16, int lo16, cudaStream_t st) {
  // vector stores: 8-channel groups start 32-byte (fp32) / 16-byte (fp16) aligned
  if ((o32 && (ld32 % 4 || (uintptr_t)o32 % 16)) ||
      (o16 && (ld16 % 8 || lo16 % 8 || (uintptr_t)o16 % 16)))
    return cudaErrorInvalidValue;
  const int gy = (co_n + kConvGroups * 8 - 1) / (kConvGroups * 8);
  const size_t tiles = (size_t)B * H * ((W + 31) / 32);
  // a few blocks per SM, each walking many pixel tiles: the weight staging is paid once
  const unsigned gx = (unsigned)std::min<size_t>(tiles, (size_t)148 * 3);
  return launch_pdl(k_conv3_small, dim3(gx, gy), dim3(32, kConvGroups), 0, st, in, wgt, bias, B, H,
                    W, co_n, act, slope, o32, ld32, o16, ld16, lo16);
}

cudaError_t launch_zero_cols_f16(__half* x, size_t rows, int c0, int ld, cudaStream_t st) {
  if (c0 >= ld) return cudaSuccess;
  return launch_pdl(k_zero_cols_f16, dim3(grid_for(rows * (ld - c0), 256)), dim3(256), 0, st, x,
                    rows, c0, ld);
}

cudaError_t launch_bicubic(const float* in, float* out, int BC, int h, int w, int oh, int ow,
                           cudaStream_t st) {
  return launch_pdl(k_bicubic, dim3(grid_for((size_t)BC * oh * ow, 256)), dim3(256), 0, st, in, out,
                    BC, h, w, oh, ow);
}

cudaError_t launch_cpb_table(const float* table, const float* w0, const float* b0, const float* w2,
                             int heads, int win, int hidden, float* out, cudaStream_t st) {
  const int total = heads * win * win * win * win;
  k_cpb_table<<<(total + 255) / 256, 256, 0, st>>>(table, w0, b0, w2, heads, win, hidden, out);
  return cudaGetLastError();
}

cudaError_t launch_up2_nhwc(const __half* in, __half* out, int B, int H, int W, int C,
                            cudaStream_t st) {
  if (C % 8) return cudaErrorInvalidValue;
  return launch_pdl(k_up2_nhwc, dim3(grid_for((size_t)B * 4 * H * W * (C / 8), 256)), dim3(256), 0,
                    st, in, out, B, H, W, C);
}

}  // namespace s2s
