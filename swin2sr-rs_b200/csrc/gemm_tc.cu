// tcgen05 GEMM and implicit-GEMM 3x3 convolution for sm_100a.
//
// One CTA computes a 128 x BN tile of D = A * B^T in TMEM (fp16 operands, fp32
// accumulation) and runs a fused epilogue on it:
//   warp 0       TMA producer: A and B K-slices (64 fp16 = one 128-byte swizzle row)
//                into a STAGES-deep shared-memory ring;
//   warp 1       allocates TMEM, issues tcgen05.mma (K = 16 per instruction) and
//                frees ring slots with tcgen05.commit;
//   warps 2..5   epilogue: tcgen05.ld of the accumulator (thread = tile row),
//                bias / activation / LayerNorm / residual in fp32, then a
//                shared-memory transpose so that every global store of a warp is
//                one contiguous row segment.
//
// In conv mode the A tile is a boxh x boxw patch of output pixels and each K-slice
// is one (tap, 64-channel chunk) of the NHWC input, fetched by a 4-D TMA box at
// the tap's offset: TMA's zero fill outside the plane IS the conv's zero padding,
// so no im2col buffer exists.
#include "common.cuh"
#include "gemm_tc.cuh"

namespace s2s {

namespace {

constexpr int kThreads = 192;
constexpr int kStageFloats = 32 * 33;  // per epilogue warp: 32 rows x 32 cols, padded

template <int BN>
struct TmemCols {
  static constexpr uint32_t value = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
};

__device__ __forceinline__ float apply_pre(const Epi& e, float v, int col) {
  if (e.bias) v += e.bias[col];
  if (e.act == ACT_GELU) {
    v = 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
  } else if (e.act == ACT_LRELU) {
    v = v < 0.0f ? v * e.slope : v;
  }
  return v;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
           const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int A_BYTES = 128 * 128;
  constexpr int B_BYTES = BN * 128;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  float* stage = reinterpret_cast<float*>(sB + STAGES * B_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(stage + 4 * kStageFloats);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accf + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t NCOLS = TmemCols<BN>::value;

  // Tile coordinates.
  const int n0 = blockIdx.y * BN;
  int m0 = 0, bimg = 0, x0 = 0, y0 = 0;
  if (!a.conv) {
    m0 = blockIdx.x * 128;
  } else {
    const int per_img = a.tiles_x * a.tiles_y;
    bimg = blockIdx.x / per_img;
    const int rem = blockIdx.x - bimg * per_img;
    y0 = (rem / a.tiles_x) * a.boxh;
    x0 = (rem % a.tiles_x) * a.boxw;
  }
  const int num_k = a.conv ? 9 * a.kc : a.K / 64;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mapA);
    tma_prefetch_desc(&mapB);
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, NCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      for (int k = 0; k < num_k; k++) {
        const int s = k % STAGES;
        if (k >= STAGES) {
          if (!mbar_wait(&empty[s], ((k / STAGES) - 1) & 1, DEV_TIMEOUT_EMPTY)) break;
        }
        mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
        if (!a.conv) {
          tma_load_2d(sA + s * A_BYTES, &mapA, &full[s], k * 64, m0);
        } else {
          const int tap = k / a.kc, cc = k - tap * a.kc;
          const int ky = tap / 3, kx = tap - ky * 3;
          tma_load_4d(sA + s * A_BYTES, &mapA, &full[s], cc * 64, x0 + kx - 1, y0 + ky - 1, bimg);
        }
        tma_load_2d(sB + s * B_BYTES, &mapB, &full[s], k * 64, n0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_f16_f32(128, BN);
      bool ok = true;
      for (int k = 0; k < num_k; k++) {
        const int s = k % STAGES;
        if (!mbar_wait(&full[s], (k / STAGES) & 1, DEV_TIMEOUT_FULL)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sw128_desc(smem_u32(sA + s * A_BYTES));
        const uint64_t bd = sw128_desc(smem_u32(sB + s * B_BYTES));
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          tc_mma_f16(tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc,
                     (k | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      (void)ok;
      tc_commit(accf);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const Epi& e = a.epi;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    int mlog, py = 0, px = 0;
    bool valid;
    if (!a.conv) {
      mlog = m0 + r;
      valid = mlog < a.M;
    } else {
      py = y0 + r / a.boxw;
      px = x0 + (r % a.boxw);
      valid = (py < a.H) && (px < a.W);
      mlog = (bimg * a.H + py) * a.W + px;
    }
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
    float* stg = stage + (warp - 2) * kStageFloats;
    const bool acc_ok = mbar_wait(accf, 0, DEV_TIMEOUT_ACC);
    tc_fence_after();

    if (acc_ok && (e.store == STORE_ROWS || e.store == STORE_SHUFFLE2)) {
      float mean = 0.0f, rstd = 1.0f;
      if (e.ln_n > 0) {
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          const int col0 = n0 + c * 32;
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int col = col0 + j;
            float x = apply_pre(e, v[j], col);
            if (e.res_pre && valid) x += e.res_pre[(size_t)mlog * e.ld_res_pre + col];
            if (col < e.ln_n) {
              s1 += x;
              s2 += x * x;
            }
          }
        }
        const float nf = (float)e.ln_n;
        mean = s1 / nf;
        const float var = fmaxf(s2 / nf - mean * mean, 0.0f);
        rstd = 1.0f / sqrtf(var + e.ln_eps);
      }
      const int F = a.N / 4;  // STORE_SHUFFLE2: output channels
#pragma unroll 1
      for (int c = 0; c < BN / 32; c++) {
        float v[32];
        tmem_ld32(tbase + c * 32, v);
        const int col0 = n0 + c * 32;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int col = col0 + j;
          float x = apply_pre(e, v[j], col);
          if (e.res_pre && valid) x += e.res_pre[(size_t)mlog * e.ld_res_pre + col];
          if (e.ln_n > 0) x = col < e.ln_n ? (x - mean) * rstd * e.ln_g[col] + e.ln_b[col] : 0.0f;
          if (col >= e.n_valid) x = 0.0f;
          stg[lane * 33 + j] = x;
        }
        __syncwarp();
        const int col = col0 + lane;
#pragma unroll 1
        for (int rr = 0; rr < 32; rr++) {
          const int m2 = __shfl_sync(0xffffffffu, mlog, rr);
          const int ok2 = __shfl_sync(0xffffffffu, (int)valid, rr);
          const int py2 = __shfl_sync(0xffffffffu, py, rr);
          const int px2 = __shfl_sync(0xffffffffu, px, rr);
          if (!ok2) continue;
          float x = stg[rr * 33 + lane];
          if (e.store == STORE_ROWS) {
            if (e.res_post) x += e.res_post[(size_t)m2 * e.ld_res_post + col];
            if (e.o32) e.o32[(size_t)(e.map32 ? e.map32[m2] : m2) * e.ld32 + col] = x;
            if (e.o32b) e.o32b[(size_t)(e.map32b ? e.map32b[m2] : m2) * e.ld32b + col] = x;
            if (e.o16)
              e.o16[(size_t)(e.map16 ? e.map16[m2] : m2) * e.ld16 + col] = __float2half_rn(x);
          } else {
            const int qd = col / F, f = col - qd * F;
            const int dy = qd >> 1, dx = qd & 1;
            const size_t dst =
                ((size_t)(bimg * 2 * a.H + 2 * py2 + dy) * (2 * a.W) + (2 * px2 + dx)) * F + f;
            if (e.res_post) x += e.res_post[dst];
            e.o16[dst] = __float2half_rn(x);
          }
        }
        __syncwarp();
      }
    } else if (acc_ok && e.store == STORE_PLANES) {
      float v[32];
      tmem_ld32(tbase, v);
      if (valid) {
        const float mean[3] = {e.mean0, e.mean1, e.mean2};
#pragma unroll
        for (int ch = 0; ch < 3; ch++) {
          const float x = apply_pre(e, v[ch], ch);
          if (e.planes_raw)
            e.planes_raw[((size_t)(bimg * 3 + ch) * a.H + py) * a.W + px] = x;
          if (e.planes && py < e.crop_h && px < e.crop_w)
            e.planes[((size_t)(bimg * 3 + ch) * e.crop_h + py) * e.crop_w + px] =
                x / e.img_range + mean[ch];
        }
      }
    } else if (acc_ok && e.store == STORE_DIRECT) {
      const float mean[3] = {e.mean0, e.mean1, e.mean2};
      const int s = e.scale, s2 = s * s, nout = 3 * s2;
#pragma unroll 1
      for (int c = 0; c < BN / 32; c++) {
        float v[32];
        tmem_ld32(tbase + c * 32, v);
        if (!valid) continue;
#pragma unroll 4
        for (int j = 0; j < 32; j++) {
          const int col = c * 32 + j;
          if (col >= nout) break;
          const int ch = col / s2, rem = col - ch * s2, dy = rem / s, dx = rem - dy * s;
          const int Y = py * s + dy, X = px * s + dx;
          if (Y < e.crop_h && X < e.crop_w)
            e.planes[((size_t)(bimg * 3 + ch) * e.crop_h + Y) * e.crop_w + X] =
                apply_pre(e, v[j], col) / e.img_range + mean[ch];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, NCOLS);
  }
}

template <int BN, int STAGES>
cudaError_t launch_t(const CUtensorMap& mapA, const CUtensorMap& mapB, const GemmArgs& a,
                     cudaStream_t st) {
  const size_t smem = 1024 + (size_t)STAGES * (128 * 128 + BN * 128) + 4 * kStageFloats * 4 +
                      (2 * STAGES + 1) * 8 + 16;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t err = cudaFuncSetAttribute(k_gemm<BN, STAGES>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    attr_set = true;
  }
  dim3 grid;
  if (a.conv)
    grid = dim3((unsigned)(a.B * a.tiles_x * a.tiles_y), (unsigned)(a.N / BN));
  else
    grid = dim3((unsigned)((a.M + 127) / 128), (unsigned)(a.N / BN));
  k_gemm<BN, STAGES><<<grid, kThreads, smem, st>>>(mapA, mapB, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm(const CUtensorMap& mapA, const CUtensorMap& mapB, const GemmArgs& a,
                        int BN, cudaStream_t st) {
  if (a.N % BN != 0 || (a.conv == 0 && a.K % 64 != 0)) return cudaErrorInvalidValue;
  if (a.epi.ln_n > 0 && a.N != BN) return cudaErrorInvalidValue;
  switch (BN) {
    case 32: return launch_t<32, 4>(mapA, mapB, a, st);
    case 64: return launch_t<64, 4>(mapA, mapB, a, st);
    case 96: return launch_t<96, 3>(mapA, mapB, a, st);
    case 128: return launch_t<128, 3>(mapA, mapB, a, st);
    case 192: return launch_t<192, 2>(mapA, mapB, a, st);
    case 256: return launch_t<256, 2>(mapA, mapB, a, st);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------- TMA maps
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}
}  // namespace

bool make_map_rows(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols_padded,
                   uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (cols_padded % 64) != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return false;
  cuuint64_t dims[2] = {cols_padded, rows};
  cuuint64_t strides[1] = {cols_padded * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_nhwc(CUtensorMap* m, const void* base, int B, int H, int W, int Cp, int boxw,
                   int boxh) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (Cp % 64) != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)Cp, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)Cp * 2, (cuuint64_t)W * Cp * 2, (cuuint64_t)H * W * Cp * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)boxw, (cuuint32_t)boxh, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void conv_box(int W, int* boxw, int* boxh) {
  int bw = 128;
  while (bw > 1 && (W % bw) != 0) bw >>= 1;
  if (bw < 8) bw = 8;  // planes are multiples of the 8-pixel window
  *boxw = bw;
  *boxh = 128 / bw;
}

}  // namespace s2s
