// Host/device interface of the tcgen05 GEMM / implicit-GEMM 3x3 convolution.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace s2s {

// ACT_QKNORM: the QKV projection's epilogue. Columns are [head][q|k|v][qk_dp]; q and k
// groups are L2-normalised per row (F.normalize, eps 1e-12) and q is further scaled by
// qk_scale[head] (the clamped logit scale times log2 e), so the attention kernel's
// logits are one dot product in the exp2 domain.
enum Act : int { ACT_NONE = 0, ACT_GELU = 1, ACT_LRELU = 2, ACT_QKNORM = 3 };

// Where the epilogue writes.
enum Store : int {
  STORE_ROWS = 0,      // row-major rows (image order), fp32 and/or fp16, by TMA bulk stores
  STORE_SHUFFLE2 = 1,  // conv output pixel-shuffled by 2 into an NHWC fp16 plane (columns
                       // ordered (dy, dx, f)), optional fp32 residual at the destination
  STORE_PLANES = 2,    // first 3 columns -> NCHW fp32 planes: denormalised+cropped and/or raw
  STORE_DIRECT = 3,    // pixelshuffledirect: column ch*s*s + dy*s + dx -> denormalised NCHW
};

struct Epi {
  const float* bias;  // padded to the full N, or null
  int act;
  float slope;
  const float* qk_scale;  // ACT_QKNORM: per head
  int qk_dp;              // ACT_QKNORM: padded head dim (16 or 32)
  // fp32 residual added after the activation (before a LayerNorm), indexed by the
  // tile's logical row and the global column; thread-per-row reads.
  const float* res_pre;
  int ld_res_pre;
  // LayerNorm over the first ln_n columns (ln_n == 0: off). Requires one N tile.
  const float* ln_g;
  const float* ln_b;
  int ln_n;
  float ln_eps;
  // fp32 residual added last (STORE_ROWS: at the logical row, brought in by TMA
  // through OutMaps::res; STORE_SHUFFLE2: at the destination pixel).
  const float* res_post;
  int ld_res_post;
  // Columns [n_valid, N) hold zeros (padded weights, bias and norms make them so).
  int n_valid;
  // Two-term fp16 output (STORE_ROWS): besides hi = fp16(v) at column n, the
  // remainder lo = fp16(v - hi) goes to column lo_off + n of the same o16 rows, so a
  // later GEMM can read both terms as one operand row [hi | lo]. 0: hi only.
  int lo_off;
  // Outputs. STORE_ROWS writes them through OutMaps (o32, o32b, o16); the pointers
  // say which are present. STORE_SHUFFLE2 writes o16 directly.
  float* o32;
  int ld32;
  float* o32b;
  int ld32b;
  __half* o16;
  int ld16;
  int store;
  // STORE_PLANES / STORE_DIRECT
  float* planes;      // denormalised, cropped to crop_h x crop_w (x scale for DIRECT)
  float* planes_raw;  // raw, uncropped [B][3][H][W]
  int crop_h, crop_w, scale;
  int crop_y0;  // plane row (x scale for DIRECT) written to output row 0
  float img_range;
  float mean0, mean1, mean2;
};

struct GemmArgs {
  int M, N, K;  // rows (GEMM mode), padded N, padded K (multiple of 64)
  int conv;     // 0: A is [M][K]; 1: A is the NHWC plane of a 3x3 convolution
  int H, W, B;  // conv plane (output geometry == input geometry)
  int boxw, boxh, tiles_x, tiles_y;
  int y_off, y_end;  // conv: output rows [y_off, y_end) of the H-row plane (rows outside
                     // are read as the 3x3 halo only)
  int kc;  // conv: 64-channel chunks per tap
  // conv with kc == 1 and boxw <= 32: mapA's boxes are (boxh + 2)-row patches, one per
  // kx, each serving its three ky taps (launch_gemm supports it for the plane store)
  int patch;
  // Two-term operands: A's K-slice for slice k (GEMM), or for chunk cc of a tap
  // (conv), is k % amod (cc % amod). With A rows [hi | lo] (amod = 2 * kc) and B
  // packed [W_hi | W_hi | W_lo] (K = 3 * kc slices), the one accumulation is
  // hi*W_hi + lo*W_hi + hi*W_lo. 0: no wrap.
  int amod;
  Epi epi;
};

// TMA descriptors of the STORE_ROWS outputs and of the post-norm residual: 32x32
// boxes (fp32 with the 128-byte swizzle, fp16 with the 64-byte swizzle), 2-D over
// [M][ld] rows in GEMM mode, 4-D over [B][H][W][ld] in conv mode (make_map_out_*).
struct OutMaps {
  CUtensorMap o32, o32b, o16, res;
};

// Launch D = A * B^T (+ epilogue). mapA / mapB are TMA descriptors built by
// make_map_* below. BN is the N tile (<= 256, multiple of 32).
cudaError_t launch_gemm(const CUtensorMap& mapA, const CUtensorMap& mapB, const OutMaps& om,
                        const GemmArgs& a, int BN, cudaStream_t st);

// Fused MLP sublayer (csrc/mlp.cu): X <- X + LN(fc2(GELU(fc1(X16)))) in place.
struct MlpArgs {
  int M;                 // tokens
  const float* b1;       // [HP] fc1 bias (padded)
  const float* b2;       // [CP] fc2 bias
  const float* g2;       // [CP] norm2 weight (zero in the pad)
  const float* beta2;    // [CP] norm2 bias
  int ln_n;              // real channels
  float ln_eps;
  float* x;              // [M][CP] fp32 residual stream, updated in place
  __half* x16;           // [M][CP] fp16 copy, updated in place
  // with the proj sublayer in front (launch_mlp's mapWp given): X <- X + LN1(proj(AO) +
  // bp), the MLP's input; then the MLP as above
  const float* bp;       // [CP] proj bias
  const float* g1;       // [CP] norm1 weight (zero in the pad)
  const float* beta1;    // [CP] norm1 bias
};

// mapX: rows map of x16 (box 128 rows); mapW1: fc1 weight [HP][CP] (box 64 rows);
// mapW2: fc2 weight [CP][HP] (box CP rows); mapX32 / mapX16o: make_map_out_rows maps of
// x (fp32) and x16. Supported (cp, hp): (192, 384), (64, 128).
// mapWp (optional, (cp, hp) = (192, 384)): proj weight [CP][CP] (box CP rows); mapX is
// then the rows map of the attention output AO, and the kernel runs proj + norm1 +
// residual first, its fp16 result staying in shared memory as fc1's operand.
cudaError_t launch_mlp(const CUtensorMap& mapX, const CUtensorMap& mapW1,
                       const CUtensorMap& mapW2, const CUtensorMap& mapX32,
                       const CUtensorMap& mapX16o, const MlpArgs& a, int cp, int hp,
                       cudaStream_t st, const CUtensorMap* mapWp = nullptr);

// Fused QKV projection + window attention (csrc/qkv_attention.cu), 6 heads x 32.
struct QaArgs {
  __half* out;        // AO rows [plane tokens][ld_out]; head h's 32 columns at h * 32
  int ld_out;
  const float* qb;    // [6][32] q bias (zero in the pad)
  const float* vb;    // [6][32] v bias (zero in the pad)
  const float* ls;    // [6] exp(min(logit_scale, ln 100)) * log2 e
  const float* bias;  // [6][576] compact position-bias table * log2 e
  int B;              // images in the plane
  int nw_img;         // windows per image (window rows x nww)
  int nww;            // windows per window row
  int wp;             // plane width
  int hp_l;           // plane rows (the output row index: (img * hp_l + y) * wp + x)
  int ghp;            // global padded rows (the shift mask's plane)
  int y_base, y_mod;  // window row wh covers plane rows (y_base + 8 wh + ty) % y_mod
  int shift;          // 0 or window / 2 (columns roll by it; the mask needs it)
  int wh_off;         // global window row of local window row 0 (band plans)
  int nwin_total;     // windows of the launch (B * nw_img)
};

// mapX: make_map_nhwc over the X16 plane with 4 x 4 boxes; mapW: Wqkv [6 x 96][192]
// (head h: rows h * 96 + q 0-31, k 32-63, v 64-95; 192-row boxes: a head pair).
cudaError_t launch_qkv_attention(const CUtensorMap& mapX, const CUtensorMap& mapW,
                                 const QaArgs& a, cudaStream_t st);
// The fused kernel's compact position-bias table from the expanded one.
cudaError_t launch_cpb_compact(const float* full, float* compact, int heads, cudaStream_t st);

// TMA descriptor helpers (driver entry point resolved at first use).
bool make_map_rows(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols_padded,
                   uint32_t box_rows);
bool make_map_nhwc(CUtensorMap* m, const void* base, int B, int H, int W, int Cp, int boxw,
                   int boxh);

// Output / residual maps (32-column boxes): rows [rows][ld] in GEMM mode, or the
// NHWC plane [B][H][W][ld] with the 32-row sub-box a warp of a conv tile owns
// (boxw = the conv tile width). elem_bytes 4 (fp32) or 2 (fp16).
bool make_map_out_rows(CUtensorMap* m, const void* base, int elem_bytes, uint64_t rows,
                       uint64_t ld);
bool make_map_out_nhwc(CUtensorMap* m, const void* base, int elem_bytes, int B, int H, int W,
                       int ld, int boxw);

// The M tile of a convolution over a W-wide plane: box width = the largest power
// of two <= 128 dividing W.
void conv_box(int W, int* boxw, int* boxh);

}  // namespace s2s
