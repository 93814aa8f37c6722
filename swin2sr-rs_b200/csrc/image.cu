// The wire format either side of the forward: PNG samples in, 8-bit RGB out.
//
// The reference's image path (src/main.rs:205-224, 365-378) is
//   load_rgb (src/image.rs:42-96)  PNG -> planar f32 in [0,1]
//   Pre::adjust (src/backend.rs:76-86)  (v - mean) * img_range
//   Backend::forward
//   Image::to_rgb8 (src/image.rs:28-39)  clamp, * 255, floor(+0.5), interleave
//   save_rgb (src/image.rs:98-114)  8-bit RGB PNG
// all on the host. Here the per-pixel steps run on the device, fused into two
// kernels either side of the forward: k_samples_in turns the decoded samples
// (8/16-bit, grey / grey+alpha / RGB / RGBA, as the png crate hands them out) into
// the mean-adjusted planar input; k_rgb8 quantises the output and optionally
// writes PNG scanlines (filter byte + filtered row, the filter chosen per row), so
// only the entropy coding is left to the host. Entropy coding is a serial
// bitstream: inflate runs on one host thread per image, deflate on several (each
// segment a raw deflate stream primed with the previous 32 KiB and ended by a sync
// flush, joined into one zlib stream with a combined Adler-32).
//
// Each float operation rounds separately (no contraction into FMA), so the device
// produces the same bytes as the reference's host arithmetic.
#include <zlib.h>

#include <algorithm>
#include <thread>

namespace s2s_image {

constexpr float kInv255 = 1.0f / 255.0f;      // src/image.rs:62 sample_scale, 8-bit
constexpr float kInv65535 = 1.0f / 65535.0f;  // src/image.rs:63 sample_scale, 16-bit

// ------------------------------------------------------------------ device kernels

// Decoded samples -> mean-adjusted planar input [B][3][h][w]. `ch` samples per
// pixel; grey (1, 2) repeats channel 0, RGB(A) takes 0..2 and ignores alpha
// (src/image.rs:83-91). 16-bit samples are big-endian byte pairs.
__global__ void k_samples_in(const uint8_t* __restrict__ s, float* __restrict__ out, int B, int h,
                             int w, int ch, int sixteen, float m0, float m1, float m2,
                             float range) {
  pdl_wait();
  const int64_t hw = (int64_t)h * w;
  const int64_t n = B * hw;
  const int bps = sixteen ? 2 : 1;
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < n;
       p += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t* px = s + p * ch * bps;
    float v[3];
    for (int c = 0; c < 3; c++) {
      const int sc = ch >= 3 ? c : 0;
      const float raw = sixteen ? (float)((px[2 * sc] << 8) | px[2 * sc + 1]) : (float)px[sc];
      v[c] = __fmul_rn(raw, sixteen ? kInv65535 : kInv255);
    }
    const int64_t b = p / hw, i = p - b * hw;
    float* o = out + b * 3 * hw + i;
    o[0] = __fmul_rn(__fsub_rn(v[0], m0), range);
    o[hw] = __fmul_rn(__fsub_rn(v[1], m1), range);
    o[2 * hw] = __fmul_rn(__fsub_rn(v[2], m2), range);
  }
  pdl_trigger();
}

// Image::to_rgb8 (src/image.rs:28-39) of one value: clamp to [0,1] (NaN stays NaN),
// * 255, + 0.5, floor, min 255 (NaN -> 255, as Rust's f32::min returns the other
// operand and `as u8` saturates).
__device__ __forceinline__ uint8_t quant8(float x) {
  if (x != x) return 255;
  const float c = fminf(fmaxf(x, 0.0f), 1.0f);
  const float v = floorf(__fadd_rn(__fmul_rn(c, 255.0f), 0.5f));
  return (uint8_t)fminf(v, 255.0f);
}

// Planar [B][3][H][W] -> interleaved [B][H][W][3] bytes.
__global__ void k_rgb8(const float* __restrict__ x, uint8_t* __restrict__ out, int B, int H,
                       int W) {
  pdl_wait();
  const int64_t hw = (int64_t)H * W, n = B * hw;
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < n;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = p / hw, i = p - b * hw;
    const float* s = x + b * 3 * hw + i;
    uint8_t* o = out + p * 3;
    o[0] = quant8(s[0]);
    o[1] = quant8(s[hw]);
    o[2] = quant8(s[2 * hw]);
  }
  pdl_trigger();
}

__device__ __forceinline__ int paeth(int a, int b, int c) {
  const int p = a + b - c, pa = abs(p - a), pb = abs(p - b), pc = abs(p - c);
  return (pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c);
}

// One PNG scanline per CTA: quantise row y and row y-1 (zeros above the first row
// of each image) into shared memory, score the five filters of the PNG
// specification by the sum of |filtered byte| read as a signed byte (the usual
// minimum-sum-of-absolute-differences heuristic; ties go to the lower type), and
// write the filter byte followed by the filtered row. Output [B][H][1 + 3W].
__global__ void __launch_bounds__(256) k_png_rows(const float* __restrict__ x,
                                                  uint8_t* __restrict__ out, int B, int H,
                                                  int W) {
  extern __shared__ uint8_t sm_rows[];
  const int L = 3 * W;
  uint8_t* cur = sm_rows;
  uint8_t* prv = sm_rows + L;
  __shared__ int part[8][5];
  __shared__ int pick;
  const int r = blockIdx.x;  // b * H + y
  const int b = r / H, y = r - b * H;
  const int64_t hw = (int64_t)H * W;
  pdl_wait();
  const float* img = x + (int64_t)b * 3 * hw;
  for (int i = threadIdx.x; i < W; i += blockDim.x) {
    for (int c = 0; c < 3; c++) {
      cur[3 * i + c] = quant8(img[c * hw + (int64_t)y * W + i]);
      prv[3 * i + c] = y > 0 ? quant8(img[c * hw + (int64_t)(y - 1) * W + i]) : 0;
    }
  }
  __syncthreads();
  int cost[5] = {0, 0, 0, 0, 0};
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    const int xv = cur[i], a = i >= 3 ? cur[i - 3] : 0, bv = prv[i], c = i >= 3 ? prv[i - 3] : 0;
    const int f[5] = {xv, xv - a, xv - bv, xv - ((a + bv) >> 1), xv - paeth(a, bv, c)};
    for (int k = 0; k < 5; k++) cost[k] += abs((int)(int8_t)(uint8_t)f[k]);
  }
  for (int k = 0; k < 5; k++)
    for (int o = 16; o; o >>= 1) cost[k] += __shfl_xor_sync(0xffffffffu, cost[k], o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0)
    for (int k = 0; k < 5; k++) part[warp][k] = cost[k];
  __syncthreads();
  if (threadIdx.x == 0) {
    int best = 0, bc = 0x7fffffff;
    for (int k = 0; k < 5; k++) {
      int t = 0;
      for (int wi = 0; wi < (int)(blockDim.x >> 5); wi++) t += part[wi][k];
      if (t < bc) bc = t, best = k;
    }
    pick = best;
  }
  __syncthreads();
  const int ft = pick;
  uint8_t* o = out + (int64_t)r * (L + 1);
  if (threadIdx.x == 0) o[0] = (uint8_t)ft;
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    const int xv = cur[i], a = i >= 3 ? cur[i - 3] : 0, bv = prv[i], c = i >= 3 ? prv[i - 3] : 0;
    const int pr = ft == 0 ? 0 : ft == 1 ? a : ft == 2 ? bv : ft == 3 ? ((a + bv) >> 1)
                                                                        : paeth(a, bv, c);
    o[1 + i] = (uint8_t)(xv - pr);
  }
  pdl_trigger();
}

}  // namespace s2s_image

namespace {

using s2s_image::k_png_rows;
using s2s_image::k_rgb8;
using s2s_image::k_samples_in;

int img_grid(int64_t n, int threads) {
  return (int)std::min<int64_t>((n + threads - 1) / threads, 148 * 16);
}

// Largest row the scanline kernel keeps in shared memory (two rows of 3W bytes).
constexpr int kPngRowsMaxSmem = 200 * 1024;

void launch_rgb8(const float* d_x, int B, int H, int W, bool png_rows, uint8_t* d_out,
                 cudaStream_t st) {
  if (!png_rows) {
    ck(launch_pdl(k_rgb8, dim3(img_grid((int64_t)B * H * W, 256)), dim3(256), 0, st, d_x, d_out, B,
                  H, W),
       "to_rgb8");
    return;
  }
  const int smem = 6 * W;
  if (smem > kPngRowsMaxSmem)
    fail(S2S_ERR_INVALID, "PNG scanlines of a " + std::to_string(W) +
                              "-pixel row exceed the kernel's shared memory");
  if (smem > 48 * 1024)
    ck(cudaFuncSetAttribute(k_png_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
       "png rows smem");
  ck(launch_pdl(k_png_rows, dim3(B * H), dim3(256), (size_t)smem, st, d_x, d_out, B, H, W),
     "png rows");
}

void check_samples(int channels, int bit_depth) {
  if (channels < 1 || channels > 4)
    fail(S2S_ERR_INVALID, "samples must have 1-4 channels (grey, grey+alpha, RGB, RGBA)");
  if (bit_depth != 8 && bit_depth != 16)
    fail(S2S_ERR_INVALID, "sample bit depth must be 8 or 16");
}

void launch_samples_in(const s2s_handle* H, int B, int h, int w, const uint8_t* d_s, int channels,
                       int bit_depth, float* d_out, cudaStream_t st) {
  const s2s_config& c = H->cfg;
  ck(launch_pdl(k_samples_in, dim3(img_grid((int64_t)B * h * w, 256)), dim3(256), 0, st, d_s, d_out,
                B, h, w, channels, bit_depth == 16 ? 1 : 0, c.mean[0], c.mean[1], c.mean[2],
                c.img_range),
     "samples in");
}

template <typename T>
void ensure_bytes(T** p, size_t* have, size_t n) {
  if (*have >= n) return;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  ck(cudaMalloc((void**)p, n * sizeof(T)), "image staging");
  *have = n;
}

// ------------------------------------------------------------------ PNG (host)
// The PNG format (ISO/IEC 15948): signature, then chunks of length / type / data /
// CRC-32; IHDR first; the image is the zlib stream split over the IDAT chunks,
// holding per scanline one filter-type byte and the filtered bytes; Adam7
// interlacing stores seven reduced images one after the other.

const uint8_t kSig[8] = {137, 80, 78, 71, 13, 10, 26, 10};

struct Png {
  uint32_t w = 0, h = 0;
  int depth = 0, ctype = 0, interlace = 0;
  int channels = 0;
  std::vector<uint8_t> idat;
  uint64_t idat_bytes = 0;  // summed IDAT chunk lengths
};

// Deflate codes at most 258 bytes of output per 2 bits of input: a zlib stream of n
// bytes inflates to less than 1032 (n + 1) bytes.
constexpr uint64_t kMaxInflateRatio = 1032;

// The filtered (with filter-type bytes) size of the image: one run per row, or per
// row of each Adam7 pass.
uint64_t raw_bytes(const Png& p);

uint32_t be32(const uint8_t* p) {
  return (uint32_t)p[0] << 24 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 8 | p[3];
}
void put32(std::vector<uint8_t>& v, uint32_t x) {
  v.push_back((uint8_t)(x >> 24));
  v.push_back((uint8_t)(x >> 16));
  v.push_back((uint8_t)(x >> 8));
  v.push_back((uint8_t)x);
}

const char* depth_name(int d) {
  switch (d) {
    case 1: return "One";
    case 2: return "Two";
    case 4: return "Four";
    case 8: return "Eight";
    default: return "Sixteen";
  }
}

// Parse the chunk stream. `want_data` false (a header query) checks only IHDR, then
// sums the IDAT chunk lengths of whatever complete chunks follow, so that a header
// whose dimensions the image data cannot possibly fill is refused before any caller
// sizes a buffer from it. Error messages for the two refusals follow
// src/image.rs:55-65, which formats the png crate's ColorType / BitDepth with {:?}.
Png parse_png(const uint8_t* d, size_t n, bool want_data) {
  if (!d || n < 8 || memcmp(d, kSig, 8) != 0) fail(S2S_ERR_INVALID, "not a PNG file (bad signature)");
  Png p;
  size_t off = 8;
  bool have_ihdr = false, done = false;
  while (!done) {
    if (n - off < 12) {
      if (have_ihdr && (!want_data || !p.idat.empty())) break;  // no IEND: what is there
      fail(S2S_ERR_INVALID, "truncated PNG chunk stream");
    }
    const uint32_t len = be32(d + off);
    const uint8_t* type = d + off + 4;
    if (have_ihdr && !want_data) {
      // header query: the rest is only measured (no CRC, no copy); a cut ends it
      if (len > 0x7fffffffu || (size_t)len > n - off - 12) break;
      if (memcmp(type, "IDAT", 4) == 0) p.idat_bytes += len;
      if (memcmp(type, "IEND", 4) == 0) break;
      off += 12 + (size_t)len;
      continue;
    }
    if (len > 0x7fffffffu || (size_t)len > n - off - 12) fail(S2S_ERR_INVALID, "truncated PNG chunk");
    const uint8_t* body = d + off + 8;
    const uint32_t crc = be32(body + len);
    if ((uint32_t)crc32(crc32(0L, Z_NULL, 0), type, len + 4) != crc)
      fail(S2S_ERR_INVALID, std::string("CRC mismatch in PNG chunk ") + std::string((const char*)type, 4));
    if (!have_ihdr) {
      if (memcmp(type, "IHDR", 4) != 0 || len != 13) fail(S2S_ERR_INVALID, "PNG does not start with IHDR");
      p.w = be32(body);
      p.h = be32(body + 4);
      p.depth = body[8];
      p.ctype = body[9];
      p.interlace = body[12];
      const int d8 = p.depth;
      bool ok = p.w > 0 && p.h > 0 && p.w <= 0x7fffffffu && p.h <= 0x7fffffffu && body[10] == 0 &&
                body[11] == 0 && p.interlace <= 1;
      switch (p.ctype) {
        case 0: ok = ok && (d8 == 1 || d8 == 2 || d8 == 4 || d8 == 8 || d8 == 16); break;
        case 3: ok = ok && (d8 == 1 || d8 == 2 || d8 == 4 || d8 == 8); break;
        case 2: case 4: case 6: ok = ok && (d8 == 8 || d8 == 16); break;
        default: ok = false;
      }
      if (!ok) fail(S2S_ERR_INVALID, "invalid PNG header");
      // at most 2^34 pixels: with <= 8 bytes a pixel every size below fits 64 bits
      if ((uint64_t)p.w * p.h > (1ull << 34)) fail(S2S_ERR_INVALID, "PNG dimensions too large");
      if (p.ctype == 3) fail(S2S_ERR_INVALID, "unsupported png colour type Indexed");
      p.channels = p.ctype == 0 ? 1 : p.ctype == 4 ? 2 : p.ctype == 2 ? 3 : 4;
      if (p.depth < 8) fail(S2S_ERR_INVALID, std::string("unsupported png bit depth ") + depth_name(p.depth));
      have_ihdr = true;
    } else if (memcmp(type, "IDAT", 4) == 0) {
      p.idat.insert(p.idat.end(), body, body + len);
      p.idat_bytes += len;
    } else if (memcmp(type, "IEND", 4) == 0) {
      done = true;
    } else if (!(type[0] & 0x20)) {
      // an unknown critical chunk (upper-case first letter) cannot be skipped
      if (memcmp(type, "PLTE", 4) != 0)
        fail(S2S_ERR_INVALID, "unknown critical PNG chunk " + std::string((const char*)type, 4));
    }
    off += 12 + (size_t)len;
  }
  if (want_data && p.idat.empty()) fail(S2S_ERR_INVALID, "PNG has no image data");
  // image data that cannot inflate to the image (only judged once some was seen)
  if (p.idat_bytes > 0 && raw_bytes(p) > kMaxInflateRatio * (p.idat_bytes + 1))
    fail(S2S_ERR_INVALID, "truncated PNG image data");
  return p;
}

struct Pass {
  int y0, x0, dy, dx;
};
const Pass kAdam7[7] = {{0, 0, 8, 8}, {0, 4, 8, 8}, {4, 0, 8, 4}, {0, 2, 4, 4},
                        {2, 0, 4, 2}, {0, 1, 2, 2}, {1, 0, 2, 1}};

inline uint32_t pass_len(uint32_t n, int o, int step) {
  return n > (uint32_t)o ? (n - o + step - 1) / step : 0;
}

inline int paeth_h(int a, int b, int c) {
  const int p = a + b - c, pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
  return (pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c);
}

// Undo the filter of one scanline in place (`prev` is the unfiltered row above, or
// null for the first row of a pass).
void unfilter(int ft, uint8_t* row, const uint8_t* prev, size_t len, int bpp) {
  switch (ft) {
    case 0: break;
    case 1: for (size_t i = bpp; i < len; i++) row[i] = (uint8_t)(row[i] + row[i - bpp]); break;
    case 2:
      if (prev) for (size_t i = 0; i < len; i++) row[i] = (uint8_t)(row[i] + prev[i]);
      break;
    case 3:
      for (size_t i = 0; i < len; i++) {
        const int a = i >= (size_t)bpp ? row[i - bpp] : 0, b = prev ? prev[i] : 0;
        row[i] = (uint8_t)(row[i] + ((a + b) >> 1));
      }
      break;
    case 4:
      for (size_t i = 0; i < len; i++) {
        const int a = i >= (size_t)bpp ? row[i - bpp] : 0, b = prev ? prev[i] : 0;
        const int c = (prev && i >= (size_t)bpp) ? prev[i - bpp] : 0;
        row[i] = (uint8_t)(row[i] + paeth_h(a, b, c));
      }
      break;
    default: fail(S2S_ERR_INVALID, "invalid PNG filter type " + std::to_string(ft));
  }
}

// Inflate + unfilter (+ de-interlace) into interleaved samples, big-endian for 16
// bits: the buffer the png crate's next_frame fills (src/image.rs:50-52).
uint64_t raw_bytes(const Png& p) {
  const uint64_t bpp = (uint64_t)p.channels * p.depth / 8;
  if (!p.interlace) return (uint64_t)p.h * ((uint64_t)p.w * bpp + 1);
  uint64_t n = 0;
  for (const Pass& q : kAdam7) {
    const uint64_t pw = pass_len(p.w, q.x0, q.dx), ph = pass_len(p.h, q.y0, q.dy);
    if (pw && ph) n += ph * (pw * bpp + 1);
  }
  return n;
}

void decode_png(const Png& p, uint8_t* out) {
  const int bpp = p.channels * p.depth / 8;
  const size_t row_bytes = (size_t)p.w * bpp;
  const size_t raw_n = (size_t)raw_bytes(p);
  std::vector<uint8_t> raw(raw_n);
  z_stream z{};
  if (inflateInit(&z) != Z_OK) fail(S2S_ERR_INVALID, "inflateInit failed");
  z.next_in = const_cast<Bytef*>(p.idat.data());
  size_t in_left = p.idat.size();
  size_t got = 0;
  int zr = Z_OK;
  while (got < raw_n) {
    const uInt in_chunk = (uInt)std::min<size_t>(in_left, 1u << 30);
    const uInt out_chunk = (uInt)std::min<size_t>(raw_n - got, 1u << 30);
    z.avail_in = in_chunk;
    z.next_out = raw.data() + got;
    z.avail_out = out_chunk;
    zr = inflate(&z, Z_NO_FLUSH);
    in_left -= in_chunk - z.avail_in;
    got += out_chunk - z.avail_out;
    if (zr == Z_STREAM_END) break;
    if (zr != Z_OK) break;
    if (in_left == 0 && z.avail_out != 0) break;
  }
  inflateEnd(&z);
  if (zr != Z_OK && zr != Z_STREAM_END && zr != Z_BUF_ERROR)
    fail(S2S_ERR_INVALID, std::string("corrupt PNG image data (zlib: ") + (z.msg ? z.msg : "error") + ")");
  if (got < raw_n) fail(S2S_ERR_INVALID, "truncated PNG image data");
  if (!p.interlace) {
    for (uint32_t y = 0; y < p.h; y++) {
      uint8_t* r = raw.data() + (size_t)y * (row_bytes + 1);
      unfilter(r[0], r + 1, y ? r - row_bytes : nullptr, row_bytes, bpp);
      memcpy(out + (size_t)y * row_bytes, r + 1, row_bytes);
    }
    return;
  }
  size_t off = 0;
  for (const Pass& q : kAdam7) {
    const size_t pw = pass_len(p.w, q.x0, q.dx), ph = pass_len(p.h, q.y0, q.dy);
    if (!pw || !ph) continue;
    const size_t pr = pw * bpp;
    for (size_t j = 0; j < ph; j++) {
      uint8_t* r = raw.data() + off + j * (pr + 1);
      unfilter(r[0], r + 1, j ? r - pr : nullptr, pr, bpp);
      const size_t y = q.y0 + j * q.dy;
      for (size_t i = 0; i < pw; i++)
        memcpy(out + y * row_bytes + (q.x0 + i * q.dx) * bpp, r + 1 + i * bpp, bpp);
    }
    off += ph * (pr + 1);
  }
}

int auto_threads(int threads) {
  if (threads > 0) return threads;
  const unsigned hc = std::thread::hardware_concurrency();
  return (int)std::max(1u, std::min(hc, 64u));
}

// Filter interleaved RGB rows on the host with the same per-row choice as
// k_png_rows, rows split over `threads`.
std::vector<uint8_t> filter_rows(int w, int h, const uint8_t* rgb, int threads) {
  const size_t L = (size_t)w * 3;
  std::vector<uint8_t> rows((size_t)h * (L + 1));
  auto work = [&](int y0, int y1) {
    for (int y = y0; y < y1; y++) {
      const uint8_t* cur = rgb + (size_t)y * L;
      const uint8_t* prv = y ? cur - L : nullptr;
      long cost[5] = {0, 0, 0, 0, 0};
      for (size_t i = 0; i < L; i++) {
        const int xv = cur[i], a = i >= 3 ? cur[i - 3] : 0, b = prv ? prv[i] : 0;
        const int c = (prv && i >= 3) ? prv[i - 3] : 0;
        const int f[5] = {xv, xv - a, xv - b, xv - ((a + b) >> 1), xv - paeth_h(a, b, c)};
        for (int k = 0; k < 5; k++) cost[k] += std::abs((int)(int8_t)(uint8_t)f[k]);
      }
      int ft = 0;
      for (int k = 1; k < 5; k++)
        if (cost[k] < cost[ft]) ft = k;
      uint8_t* o = rows.data() + (size_t)y * (L + 1);
      o[0] = (uint8_t)ft;
      for (size_t i = 0; i < L; i++) {
        const int a = i >= 3 ? cur[i - 3] : 0, b = prv ? prv[i] : 0;
        const int c = (prv && i >= 3) ? prv[i - 3] : 0;
        const int pr = ft == 0 ? 0 : ft == 1 ? a : ft == 2 ? b : ft == 3 ? ((a + b) >> 1)
                                                                           : paeth_h(a, b, c);
        o[1 + i] = (uint8_t)(cur[i] - pr);
      }
    }
  };
  const int T = std::max(1, std::min(auto_threads(threads), h / 16 + 1));
  std::vector<std::thread> ts;
  for (int t = 0; t < T; t++) ts.emplace_back(work, (int)((int64_t)h * t / T), (int)((int64_t)h * (t + 1) / T));
  for (auto& t : ts) t.join();
  return rows;
}

// One zlib stream of `data` compressed in parallel: segment k is a raw deflate
// stream primed with the 32 KiB before it (deflateSetDictionary) and closed by
// Z_SYNC_FLUSH, the last by Z_FINISH; their concatenation is one valid deflate
// stream. Header and the Adler-32 trailer (adler32_combine) wrap it.
std::vector<uint8_t> zlib_parallel(const uint8_t* data, size_t n, int level, int threads) {
  const int T = auto_threads(threads);
  const size_t seg = std::max<size_t>(256 * 1024, (n + T - 1) / T);
  const size_t nseg = std::max<size_t>(1, (n + seg - 1) / seg);
  std::vector<std::vector<uint8_t>> parts(nseg);
  std::vector<uLong> adl(nseg);
  std::vector<std::string> errs(nseg);
  auto work = [&](size_t k) {
    const size_t a = k * seg, b = std::min(n, a + seg);
    z_stream z{};
    if (deflateInit2(&z, level, Z_DEFLATED, -15, 8, Z_DEFAULT_STRATEGY) != Z_OK) {
      errs[k] = "deflateInit2 failed";
      return;
    }
    if (a > 0) {
      const size_t dict = std::min<size_t>(a, 32768);
      deflateSetDictionary(&z, data + a - dict, (uInt)dict);
    }
    std::vector<uint8_t>& out = parts[k];
    out.resize(deflateBound(&z, (uLong)(b - a)) + 64);
    z.next_in = const_cast<Bytef*>(data + a);
    z.avail_in = (uInt)(b - a);
    z.next_out = out.data();
    z.avail_out = (uInt)out.size();
    const bool last = k + 1 == nseg;
    const int r = deflate(&z, last ? Z_FINISH : Z_SYNC_FLUSH);
    if ((last && r != Z_STREAM_END) || (!last && (r != Z_OK || z.avail_in != 0)))
      errs[k] = "deflate failed";
    out.resize(out.size() - z.avail_out);
    deflateEnd(&z);
    adl[k] = adler32(adler32(0L, Z_NULL, 0), data + a, (uInt)(b - a));
  };
  std::vector<std::thread> ts;
  for (size_t k = 1; k < nseg; k++) ts.emplace_back(work, k);
  work(0);
  for (auto& t : ts) t.join();
  for (auto& e : errs)
    if (!e.empty()) fail(S2S_ERR_INVALID, e);
  std::vector<uint8_t> z;
  const int flevel = level < 0 ? 2 : level < 2 ? 0 : level < 6 ? 1 : level == 6 ? 2 : 3;
  const unsigned cmf = 0x78, flg0 = (unsigned)flevel << 6;
  z.push_back((uint8_t)cmf);
  z.push_back((uint8_t)(flg0 + (31 - (cmf * 256 + flg0) % 31) % 31));
  uLong ad = adler32(0L, Z_NULL, 0);
  for (size_t k = 0; k < nseg; k++) {
    z.insert(z.end(), parts[k].begin(), parts[k].end());
    const size_t a = k * seg, b = std::min(n, a + seg);
    ad = adler32_combine(ad, adl[k], (z_off_t)(b - a));
  }
  put32(z, (uint32_t)ad);
  return z;
}

void put_chunk(std::vector<uint8_t>& f, const char* type, const uint8_t* body, size_t len) {
  put32(f, (uint32_t)len);
  const size_t at = f.size();
  f.insert(f.end(), type, type + 4);
  if (len) f.insert(f.end(), body, body + len);
  put32(f, (uint32_t)crc32(crc32(0L, Z_NULL, 0), f.data() + at, (uInt)(len + 4)));
}

// An 8-bit RGB PNG around already-filtered scanlines (src/image.rs:105-114 writes
// the same colour type and depth).
std::vector<uint8_t> png_from_rows(int w, int h, const uint8_t* rows, int level, int threads) {
  const size_t L = (size_t)w * 3 + 1;
  for (int y = 0; y < h; y++)
    if (rows[(size_t)y * L] > 4)
      fail(S2S_ERR_INVALID, "scanline " + std::to_string(y) + " has filter type " +
                                std::to_string(rows[(size_t)y * L]) + " (0-4 allowed)");
  std::vector<uint8_t> z = zlib_parallel(rows, (size_t)h * L, level, threads);
  std::vector<uint8_t> f(kSig, kSig + 8);
  uint8_t ihdr[13];
  const uint32_t ww = (uint32_t)w, hh = (uint32_t)h;
  for (int i = 0; i < 4; i++) {
    ihdr[i] = (uint8_t)(ww >> (24 - 8 * i));
    ihdr[4 + i] = (uint8_t)(hh >> (24 - 8 * i));
  }
  ihdr[8] = 8;   // bit depth
  ihdr[9] = 2;   // RGB
  ihdr[10] = 0;  // deflate
  ihdr[11] = 0;  // adaptive filtering
  ihdr[12] = 0;  // not interlaced
  put_chunk(f, "IHDR", ihdr, 13);
  const size_t kIdat = 1 << 20;
  for (size_t o = 0; o < z.size(); o += kIdat)
    put_chunk(f, "IDAT", z.data() + o, std::min(kIdat, z.size() - o));
  put_chunk(f, "IEND", nullptr, 0);
  return f;
}

template <typename F>
int guarded_free(F&& f) {
  try {
    f();
    return S2S_OK;
  } catch (const S2SError& e) {
    g_create_error = e.msg;
    return e.code;
  } catch (const std::bad_alloc&) {
    g_create_error = "host allocation failed";
    return S2S_ERR_OOM;
  }
}

int export_buffer(const std::vector<uint8_t>& f, uint8_t** png, size_t* bytes) {
  uint8_t* p = static_cast<uint8_t*>(malloc(f.size()));
  if (!p) {
    g_create_error = "host allocation failed";
    return S2S_ERR_OOM;
  }
  memcpy(p, f.data(), f.size());
  *png = p;
  *bytes = f.size();
  return S2S_OK;
}

}  // namespace

extern "C" {

int s2s_png_header(const void* png, size_t bytes, int* width, int* height, int* channels,
                   int* bit_depth) {
  return guarded_free([&] {
    const Png p = parse_png(static_cast<const uint8_t*>(png), bytes, false);
    if (width) *width = (int)p.w;
    if (height) *height = (int)p.h;
    if (channels) *channels = p.channels;
    if (bit_depth) *bit_depth = p.depth;
  });
}

int s2s_png_decode(const void* png, size_t bytes, void* samples, size_t capacity) {
  return guarded_free([&] {
    const Png p = parse_png(static_cast<const uint8_t*>(png), bytes, true);
    const size_t need = (size_t)p.w * p.h * p.channels * (p.depth / 8);
    if (!samples || capacity < need)
      fail(S2S_ERR_INVALID, "sample buffer holds " + std::to_string(capacity) + " bytes, the image needs " +
                                std::to_string(need));
    decode_png(p, static_cast<uint8_t*>(samples));
  });
}

int s2s_png_encode_rgb8(int width, int height, const uint8_t* rgb, int level, int threads,
                        uint8_t** png, size_t* bytes) {
  if (!png || !bytes) return S2S_ERR_INVALID;
  std::vector<uint8_t> f;
  const int rc = guarded_free([&] {
    if (width < 1 || height < 1 || !rgb) fail(S2S_ERR_INVALID, "s2s_png_encode_rgb8: empty image");
    if (level < -1 || level > 9) fail(S2S_ERR_INVALID, "compression level must be -1..9");
    f = png_from_rows(width, height, filter_rows(width, height, rgb, threads).data(), level, threads);
  });
  return rc != S2S_OK ? rc : export_buffer(f, png, bytes);
}

int s2s_png_encode_rows(int width, int height, const uint8_t* rows, int level, int threads,
                        uint8_t** png, size_t* bytes) {
  if (!png || !bytes) return S2S_ERR_INVALID;
  std::vector<uint8_t> f;
  const int rc = guarded_free([&] {
    if (width < 1 || height < 1 || !rows) fail(S2S_ERR_INVALID, "s2s_png_encode_rows: empty image");
    if (level < -1 || level > 9) fail(S2S_ERR_INVALID, "compression level must be -1..9");
    f = png_from_rows(width, height, rows, level, threads);
  });
  return rc != S2S_OK ? rc : export_buffer(f, png, bytes);
}

void s2s_free(void* p) { free(p); }

int s2s_adjust_device(const s2s_handle* H, int batch, int height, int width, const void* d_samples,
                      int channels, int bit_depth, float* d_chw, void* stream) {
  if (!H || !d_samples || !d_chw) return S2S_ERR_INVALID;
  s2s_handle* M = const_cast<s2s_handle*>(H);
  return guarded(M, [&] {
    check_samples(channels, bit_depth);
    if (batch < 1 || height < 1 || width < 1) fail(S2S_ERR_INVALID, "empty image");
    launch_samples_in(H, batch, height, width, static_cast<const uint8_t*>(d_samples), channels,
                      bit_depth, d_chw, stream ? (cudaStream_t)stream : H->stream);
  });
}

int s2s_rgb8_device(int batch, int height, int width, const float* d_chw, int png_rows,
                    uint8_t* d_out, void* stream) {
  if (!d_chw || !d_out) return S2S_ERR_INVALID;
  return guarded_free([&] {
    if (batch < 1 || height < 1 || width < 1) fail(S2S_ERR_INVALID, "empty image");
    launch_rgb8(d_chw, batch, height, width, png_rows != 0, d_out, (cudaStream_t)stream);
  });
}

int s2s_forward_image(s2s_handle* H, int batch, int height, int width, const void* samples,
                      int channels, int bit_depth, int png_rows, uint8_t* out, uint8_t* aux) {
  if (!H || !samples || !out) return S2S_ERR_INVALID;
  return guarded(H, [&] {
    if (H->band_world > 1) fail(S2S_ERR_INVALID, kBandHandle);
    check_samples(channels, bit_depth);
    if (batch < 1) fail(S2S_ERR_INVALID, "batch must be >= 1");
    const int win = H->cfg.window, s = H->cfg.scale;
    const int hp = (height / win + 1) * win, wp = (width / win + 1) * win;
    const size_t nin = (size_t)batch * height * width * channels * (bit_depth / 8);
    const size_t nout = (size_t)batch * 3 * height * s * width * s;
    const size_t naux = (size_t)batch * 3 * hp * wp;
    const bool has_aux = H->cfg.upsampler == S2S_PIXELSHUFFLE_AUX;
    const size_t out_b = png_rows ? (size_t)batch * height * s * (3 * (size_t)width * s + 1) : nout;
    const size_t aux_b = png_rows ? (size_t)batch * hp * (3 * (size_t)wp + 1) : naux;
    const size_t tot_b = out_b + (has_aux && aux ? aux_b : 0);
    ensure_bytes(&H->b_in, &H->b_in_n, nin);
    ensure_bytes(&H->b_out, &H->b_out_n, tot_b);
    ensure_staging(H, &H->h_in, &H->h_in_n, (size_t)batch * 3 * height * width);
    ensure_staging(H, &H->h_out, &H->h_out_n, nout);
    if (has_aux) ensure_staging(H, &H->h_aux, &H->h_aux_n, naux);
    cudaStream_t st = H->stream;
    ck(cudaMemcpyAsync(H->b_in, samples, nin, cudaMemcpyHostToDevice, st), "upload");
    launch_samples_in(H, batch, height, width, H->b_in, channels, bit_depth, H->h_in, st);
    H->launches++;
    run_forward(H, batch, height, width, H->h_in, H->h_out, has_aux ? H->h_aux : nullptr, st);
    launch_rgb8(H->h_out, batch, height * s, width * s, png_rows != 0, H->b_out, st);
    H->launches++;
    if (has_aux && aux) {
      launch_rgb8(H->h_aux, batch, hp, wp, png_rows != 0, H->b_out + out_b, st);
      H->launches++;
    }
    ck(cudaMemcpyAsync(out, H->b_out, out_b, cudaMemcpyDeviceToHost, st), "download");
    if (has_aux && aux)
      ck(cudaMemcpyAsync(aux, H->b_out + out_b, aux_b, cudaMemcpyDeviceToHost, st), "download");
    ck(cudaStreamSynchronize(st), "forward");
    check_device_error(H);
    if (H->profiling) drain_profile(H);
  });
}

}  // extern "C"
