// CPU ORACLE - TEST INFRASTRUCTURE ONLY.
//
// A restatement, in C++, of the reference's CPU forward pass (swin2sr-rs
// src/cpu.rs + src/plan.rs). It is the checker the CUDA path is held to and the
// timed CPU baseline; nothing in the product links or calls it. Only tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline / --impl reference legs load
// this library.
//
// Parity pin: the forward is checked against the published PyTorch network
// (tools/network_swin2sr.py) on seeded weights through the SW2F fixtures under
// tests/golden/ (made by tests/golden/make_golden.py), and the bicubic resample
// against the reference's own golden vectors (tests/bicubic.rs:38-58 data).
//
// Arithmetic follows the reference op by op, with the same summation orders and
// no fused multiply-add (built with -ffp-contract=off, as Rust computes `a += w * x`
// as a multiply then an add):
//   conv3x3            lightgpu conv3x3s1p1 as documented at src/cpu.rs:378-414:
//                      bias first, taps ky, kx, ci, missing edge taps skipped
//   conv_row/_shuffle2 src/cpu.rs:431-542: bias first, ci, ky, kx
//   conv1x1 / linear   src/cpu.rs:544-577, 607-775: bias first, ci ascending
//   channel_layer_norm src/cpu.rs:1019-1073: one-pass s1, s2 ascending channel,
//                      var = s2/n - mean^2 clamped at 0, eps 1e-5
//   attention          src/cpu.rs:1244-1402: dot/(qn*kn) * exp(min(ls, ln 100)) + cpb,
//                      -100 across regions, max-subtracted softmax with fast_exp
//   fast_exp           src/cpu.rs:1095-1120 (the reference's own polynomial)
//   gelu               src/cpu.rs:1125-1132 (erf form; lightgpu's erf is not
//                      vendored, so libm erff stands in)
//   bicubic_resize     src/cpu.rs:877-935
//   forward / head     src/cpu.rs:1437-1880, finish / finish_aux :1892-1941
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

const float LN_EPS = 1e-5f;

struct Net {
  int ups;  // 0 pixelshuffle, 1 pixelshuffledirect, 2 nearest+conv, 3 pixelshuffle_aux
  int scale, win, c, heads, hd, mlp;
  std::vector<int> depths;
  float img_range, mean[3];
  std::map<std::string, const float*> t;
  std::map<std::string, int64_t> n;
  const float* w(const std::string& k) const {
    auto it = t.find(k);
    return it == t.end() ? nullptr : it->second;
  }
};

struct Plan {
  int h, w, hp, wp, win, nwh, nww, nw, n, c;
  Plan(int h_, int w_, int win_, int c_) : h(h_), w(w_), win(win_), c(c_) {
    hp = (h / win + 1) * win;
    wp = (w / win + 1) * win;
    nwh = hp / win;
    nww = wp / win;
    nw = nwh * nww;
    n = win * win;
  }
  int tokens() const { return nw * n; }
  int plane() const { return hp * wp; }
  int shift_for(int b) const { return (b % 2 == 1) ? win / 2 : 0; }
  // src/plan.rs:72-78
  void index(int wi, int t, int shift, int& a, int& b) const {
    int wh = wi / nww, ww = wi % nww, i = t / win, j = t % win;
    a = (wh * win + i + shift) % hp;
    b = (ww * win + j + shift) % wp;
  }
};

// src/plan.rs:95-105
int region_of(int a, int p, int win, int shift) {
  if (a + win < p) return 0;
  if (a + shift < p) return 1;
  return 2;
}

// src/plan.rs:116-139: rows first, then columns, whole-plane mirror.
std::vector<float> pad_reflect(const float* x, int c, int h, int w, int hp, int wp) {
  std::vector<float> rows((size_t)c * hp * w), out((size_t)c * hp * wp);
  for (int ch = 0; ch < c; ch++)
    for (int y = 0; y < hp; y++) {
      int sy = y < h ? y : 2 * h - 1 - std::min(y, 2 * h - 1);
      memcpy(&rows[((size_t)ch * hp + y) * w], &x[((size_t)ch * h + sy) * w], sizeof(float) * w);
    }
  for (int ch = 0; ch < c; ch++)
    for (int y = 0; y < hp; y++)
      for (int bx = 0; bx < wp; bx++) {
        int sx = bx < w ? bx : 2 * w - 1 - std::min(bx, 2 * w - 1);
        out[((size_t)ch * hp + y) * wp + bx] = rows[((size_t)ch * hp + y) * w + sx];
      }
  return out;
}

// 3x3 s1 p1, NCHW: out[co][y][x] = b[co] + sum_{ky,kx,ci} w*in (taps off the plane skipped).
void conv3x3(const float* in, int ci_n, int h, int w, const float* wgt, int co_n,
             const float* bias, float* out) {
  const int CB = 8;
  int nco = (co_n + CB - 1) / CB;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
  for (int y = 0; y < h; y++)
    for (int cb = 0; cb < nco; cb++) {
      int co0 = cb * CB, co1 = std::min(co_n, co0 + CB);
      std::vector<float> acc((size_t)CB * w);
      for (int co = co0; co < co1; co++)
        for (int x = 0; x < w; x++) acc[(size_t)(co - co0) * w + x] = bias[co];
      for (int ky = 0; ky < 3; ky++) {
        int sy = y + ky - 1;
        if (sy < 0 || sy >= h) continue;
        for (int kx = 0; kx < 3; kx++) {
          int x0 = kx == 0 ? 1 : 0, x1 = kx == 2 ? w - 1 : w;
          for (int ci = 0; ci < ci_n; ci++) {
            const float* src = in + ((size_t)ci * h + sy) * w + (kx - 1);
            for (int co = co0; co < co1; co++) {
              float wv = wgt[(((size_t)co * ci_n + ci) * 3 + ky) * 3 + kx];
              float* d = &acc[(size_t)(co - co0) * w];
              for (int x = x0; x < x1; x++) d[x] += wv * src[x];
            }
          }
        }
      }
      for (int co = co0; co < co1; co++)
        memcpy(out + ((size_t)co * h + y) * w, &acc[(size_t)(co - co0) * w], sizeof(float) * w);
    }
}

// src/cpu.rs:431-480 conv_row: dest = b; for ci, for ky in range, kx 0..2.
void conv_row(const float* in, int ci_n, int h, int w, const float* wc, float b, int y,
              float* dest) {
  for (int x = 0; x < w; x++) dest[x] = b;
  int ky0 = y == 0 ? 1 : 0, ky1 = (y + 1 == h) ? 1 : 2;
  size_t hw = (size_t)h * w;
  for (int ci = 0; ci < ci_n; ci++) {
    const float* ic = in + ci * hw;
    const float* k = wc + ci * 9;
    for (int ky = ky0; ky <= ky1; ky++) {
      const float* srow = ic + (size_t)(y + ky - 1) * w;
      const float* kr = k + ky * 3;
      if (w == 1) {
        dest[0] += kr[1] * srow[0];
        continue;
      }
      dest[0] += kr[1] * srow[0];
      dest[0] += kr[2] * srow[1];
      for (int x = 1; x < w - 1; x++) {
        dest[x] += kr[0] * srow[x - 1];
        dest[x] += kr[1] * srow[x];
        dest[x] += kr[2] * srow[x + 1];
      }
      dest[w - 1] += kr[0] * srow[w - 2];
      dest[w - 1] += kr[1] * srow[w - 1];
    }
  }
}

// src/cpu.rs:498-542: conv straight into the pixel-shuffled layout, out [feat][2h][2w].
void conv3x3_shuffle2(const float* in, int ci_n, int h, int w, const float* wgt, int feat,
                      const float* bias, float* out) {
  int h2 = 2 * h, w2 = 2 * w;
#pragma omp parallel
  {
    std::vector<float> t0(w), t1(w);
#pragma omp for schedule(dynamic, 8)
    for (int i = 0; i < feat * h2; i++) {
      int ch = i / h2, y2 = i % h2, dy = y2 % 2, y = y2 / 2;
      int co0 = 4 * ch + 2 * dy, co1 = co0 + 1;
      conv_row(in, ci_n, h, w, wgt + (size_t)co0 * ci_n * 9, bias[co0], y, t0.data());
      conv_row(in, ci_n, h, w, wgt + (size_t)co1 * ci_n * 9, bias[co1], y, t1.data());
      float* dest = out + (size_t)i * w2;
      for (int x = 0; x < w; x++) {
        dest[2 * x] = t0[x];
        dest[2 * x + 1] = t1[x];
      }
    }
  }
}

// out[r][co] = bias[co] + sum_ci w[co][ci] x[r][ci], ci ascending (src/cpu.rs:607-775).
void linear(const float* x, int rows, int ci_n, const float* wgt, int co_n, const float* bias,
            float* out) {
  std::vector<float> wt((size_t)ci_n * co_n);
  for (int co = 0; co < co_n; co++)
    for (int ci = 0; ci < ci_n; ci++) wt[(size_t)ci * co_n + co] = wgt[(size_t)co * ci_n + ci];
  const int MR = 8;
  int nb = (rows + MR - 1) / MR;
#pragma omp parallel
  {
    std::vector<float> acc((size_t)MR * co_n);
#pragma omp for schedule(static)
    for (int rb = 0; rb < nb; rb++) {
      int r0 = rb * MR, r1 = std::min(rows, r0 + MR);
      for (int r = r0; r < r1; r++)
        for (int co = 0; co < co_n; co++)
          acc[(size_t)(r - r0) * co_n + co] = bias ? bias[co] : 0.0f;
      for (int ci = 0; ci < ci_n; ci++) {
        const float* wr = &wt[(size_t)ci * co_n];
        for (int r = r0; r < r1; r++) {
          float xv = x[(size_t)r * ci_n + ci];
          float* a = &acc[(size_t)(r - r0) * co_n];
          for (int co = 0; co < co_n; co++) a[co] += wr[co] * xv;
        }
      }
      for (int r = r0; r < r1; r++)
        memcpy(out + (size_t)r * co_n, &acc[(size_t)(r - r0) * co_n], sizeof(float) * co_n);
    }
  }
}

// 1x1 conv over an NCHW plane, bias first, ci ascending (src/cpu.rs:544-577).
void conv1x1(const float* in, int ci_n, int hw, const float* wgt, int co_n, const float* bias,
             float* out) {
#pragma omp parallel for schedule(static)
  for (int co = 0; co < co_n; co++) {
    float* d = out + (size_t)co * hw;
    for (int p = 0; p < hw; p++) d[p] = bias[co];
    for (int ci = 0; ci < ci_n; ci++) {
      float wv = wgt[(size_t)co * ci_n + ci];
      const float* s = in + (size_t)ci * hw;
      for (int p = 0; p < hw; p++) d[p] += wv * s[p];
    }
  }
}

// src/cpu.rs:1019-1073 (one-pass statistics, ascending channel order).
void channel_layer_norm(const float* x, const float* w, const float* b, float* y, int c,
                        int hw) {
  std::vector<float> s1(hw, 0.0f), s2(hw, 0.0f);
  const int BLK = 64;
#pragma omp parallel for schedule(static)
  for (int p0 = 0; p0 < hw; p0 += BLK) {
    int p1 = std::min(hw, p0 + BLK);
    for (int ch = 0; ch < c; ch++) {
      const float* pl = x + (size_t)ch * hw;
      for (int p = p0; p < p1; p++) {
        float v = pl[p];
        s1[p] += v;
        s2[p] += v * v;
      }
    }
  }
  float nf = (float)c;
  std::vector<float> mean(hw), rstd(hw);
  for (int p = 0; p < hw; p++) {
    float m = s1[p] / nf;
    float var = s2[p] / nf - m * m;
    mean[p] = m;
    rstd[p] = 1.0f / std::sqrt(std::max(var, 0.0f) + LN_EPS);
  }
#pragma omp parallel for schedule(static)
  for (int ch = 0; ch < c; ch++) {
    const float* pl = x + (size_t)ch * hw;
    float* d = y + (size_t)ch * hw;
    float wv = w[ch], bv = b[ch];
    for (int p = 0; p < hw; p++) d[p] = (pl[p] - mean[p]) * rstd[p] * wv + bv;
  }
}

// src/cpu.rs:1095-1120.
float fast_exp(float x) {
  const float LOG2_E = 1.4426950408889634f;
  float t = x * LOG2_E;
  float n = std::floor(t + 0.5f) - 0.5f;
  if (n < -126.0f) return 0.0f;
  float f = t - n;
  float p = 1.0f + f * (0.69314718f +
                        f * (0.24022651f +
                             f * (0.05550411f +
                                  f * (0.009618129f + f * (0.0013333558f + f * 0.0001540353f)))));
  // `n as i32` in Rust truncates toward zero, as the C cast does.
  uint32_t bits = (uint32_t)(((int32_t)n) + 127) << 23;
  float scale;
  memcpy(&scale, &bits, 4);
  return scale * p;
}

void gelu_erf_inplace(float* x, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; i++) {
    float v = x[i];
    x[i] = 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
  }
}

// src/cpu.rs:1148-1222: plane [c][hp][wp] <-> window-major tokens [nw*n][c].
void gather(const Plan& pl, const float* x, int shift, float* tok) {
  int c = pl.c;
  size_t hw = (size_t)pl.hp * pl.wp;
#pragma omp parallel for schedule(static)
  for (int wi = 0; wi < pl.nw; wi++)
    for (int t = 0; t < pl.n; t++) {
      int y, xx;
      pl.index(wi, t, shift, y, xx);
      size_t p = (size_t)y * pl.wp + xx;
      float* d = tok + ((size_t)wi * pl.n + t) * c;
      for (int i = 0; i < c; i++) d[i] = x[i * hw + p];
    }
}

void scatter(const Plan& pl, const float* tok, int shift, float* x) {
  int c = pl.c;
  size_t hw = (size_t)pl.hp * pl.wp;
#pragma omp parallel for schedule(static)
  for (int wi = 0; wi < pl.nw; wi++)
    for (int t = 0; t < pl.n; t++) {
      int y, xx;
      pl.index(wi, t, shift, y, xx);
      size_t p = (size_t)y * pl.wp + xx;
      const float* s = tok + ((size_t)wi * pl.n + t) * c;
      for (int i = 0; i < c; i++) x[i * hw + p] = s[i];
    }
}

// src/cpu.rs:1244-1402. qkv is [3][tokens][c]; out is [tokens][c].
void attention(const Plan& pl, int heads, int hdim, const float* logit_scale, const float* cpb,
               const float* qkv, int shift, float* out) {
  int c = pl.c, n = pl.n;
  size_t tok_c = (size_t)pl.tokens() * c;
  bool masked = shift != 0;
  std::vector<float> ls(heads);
  for (int h = 0; h < heads; h++) ls[h] = std::exp(std::min(logit_scale[h], std::log(100.0f)));
  std::vector<float> cpbt((size_t)heads * n * n);
  for (int q = 0; q < n; q++)
    for (int k = 0; k < n; k++)
      for (int h = 0; h < heads; h++)
        cpbt[((size_t)h * n + q) * n + k] = cpb[((size_t)q * n + k) * heads + h];
#pragma omp parallel
  {
    std::vector<float> scores(n), kn(n);
    std::vector<size_t> ktok(n);
    std::vector<int> kreg0(n), kreg1(n);
#pragma omp for schedule(dynamic, 4)
    for (int wi = 0; wi < pl.nw; wi++) {
      float* outw = out + (size_t)wi * n * c;
      int wh = wi / pl.nww, ww = wi % pl.nww;
      for (int k = 0; k < n; k++) {
        ktok[k] = (size_t)wi * n + k;
        if (masked) {
          int i = k / pl.win, j = k % pl.win;
          kreg0[k] = region_of(wh * pl.win + i, pl.hp, pl.win, shift);
          kreg1[k] = region_of(ww * pl.win + j, pl.wp, pl.win, shift);
        }
      }
      for (int hh = 0; hh < heads; hh++) {
        int off = hh * hdim;
        for (int k = 0; k < n; k++) {
          const float* kv = qkv + tok_c + ktok[k] * c + off;
          float s = 0.0f;
          for (int d = 0; d < hdim; d++) s += kv[d] * kv[d];
          kn[k] = std::max(std::sqrt(s), 1e-12f);
        }
        for (int q = 0; q < n; q++) {
          float* orow = outw + (size_t)q * c;
          const float* qv = qkv + ktok[q] * c + off;
          float qs = 0.0f;
          for (int d = 0; d < hdim; d++) qs += qv[d] * qv[d];
          float qn = std::max(std::sqrt(qs), 1e-12f);
          for (int k = 0; k < n; k++) {
            const float* kv = qkv + tok_c + ktok[k] * c + off;
            float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
            int d = 0;
            for (; d + 4 <= hdim; d += 4) {
              a0 += qv[d] * kv[d];
              a1 += qv[d + 1] * kv[d + 1];
              a2 += qv[d + 2] * kv[d + 2];
              a3 += qv[d + 3] * kv[d + 3];
            }
            float tail = 0;
            for (; d < hdim; d++) tail += qv[d] * kv[d];
            float dot = ((a0 + a1) + (a2 + a3) + tail) / (qn * kn[k]);
            float s = dot * ls[hh] + cpbt[((size_t)hh * n + q) * n + k];
            if (masked && (kreg0[q] != kreg0[k] || kreg1[q] != kreg1[k])) s -= 100.0f;
            scores[k] = s;
          }
          float mx = -INFINITY;
          for (int k = 0; k < n; k++) mx = std::max(mx, scores[k]);
          float sum = 0;
          for (int k = 0; k < n; k++) {
            scores[k] = fast_exp(scores[k] - mx);
            sum += scores[k];
          }
          float inv = 1.0f / sum;
          const float* vb = qkv + 2 * tok_c + off;
          for (int d = 0; d < hdim; d++) {
            float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
            int k = 0;
            for (; k + 4 <= n; k += 4) {
              a0 += scores[k] * vb[ktok[k] * c + d];
              a1 += scores[k + 1] * vb[ktok[k + 1] * c + d];
              a2 += scores[k + 2] * vb[ktok[k + 2] * c + d];
              a3 += scores[k + 3] * vb[ktok[k + 3] * c + d];
            }
            float tail = 0;
            for (; k < n; k++) tail += scores[k] * vb[ktok[k] * c + d];
            orow[off + d] = ((a0 + a1) + (a2 + a3) + tail) * inv;
          }
        }
      }
    }
  }
}

void leaky_relu(float* x, size_t n, float slope) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; i++)
    if (x[i] < 0.0f) x[i] *= slope;
}

void add_into(const float* a, float* y, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; i++) y[i] += a[i];
}

// src/cpu.rs:814-849
void pixel_shuffle(const float* in, int c, int h, int w, int s, float* out) {
  int oh = h * s, ow = w * s;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < c * oh; r++) {
    int ch = r / oh, rem = r % oh, dy = rem % s, y = rem / s;
    float* dst = out + (size_t)r * ow;
    for (int dx = 0; dx < s; dx++) {
      const float* src = in + (((size_t)ch * s * s + dy * s + dx) * h + y) * w;
      for (int x = 0; x < w; x++) dst[x * s + dx] = src[x];
    }
  }
}

// src/cpu.rs:877-935: torch bicubic (a = -0.75), align_corners=False, edge clamp.
float cubic_w(float t) {
  const float A = -0.75f;
  t = std::fabs(t);
  if (t <= 1.0f) return ((A + 2.0f) * t - (A + 3.0f)) * t * t + 1.0f;
  if (t < 2.0f) return (((t - 5.0f) * t + 8.0f) * t - 4.0f) * A;
  return 0.0f;
}

void bicubic_taps(int n_in, int n_out, std::vector<int>& idx, std::vector<float>& wt) {
  idx.resize((size_t)n_out * 4);
  wt.resize((size_t)n_out * 4);
  for (int i = 0; i < n_out; i++) {
    float src = ((float)i + 0.5f) * ((float)n_in / (float)n_out) - 0.5f;
    float base = std::floor(src);
    for (int m = 0; m < 4; m++) {
      long ix = (long)base - 1 + m;
      ix = std::min<long>(std::max<long>(ix, 0), n_in - 1);
      idx[i * 4 + m] = (int)ix;
      wt[i * 4 + m] = cubic_w(src - (base + (float)m - 1.0f));
    }
  }
}

void bicubic_resize(const float* in, int c, int h, int w, int oh, int ow, float* out) {
  std::vector<int> iy, ix;
  std::vector<float> wy, wx;
  bicubic_taps(h, oh, iy, wy);
  bicubic_taps(w, ow, ix, wx);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < c * oh; i++) {
    int ch = i / oh, y = i % oh;
    const float* src = in + (size_t)ch * h * w;
    float* dst = out + (size_t)i * ow;
    for (int x = 0; x < ow; x++) {
      float acc = 0.0f;
      for (int m = 0; m < 4; m++) {
        const float* r = src + (size_t)iy[y * 4 + m] * w;
        float a0 = wx[x * 4 + 0] * r[ix[x * 4 + 0]];
        float a1 = wx[x * 4 + 1] * r[ix[x * 4 + 1]];
        float a2 = wx[x * 4 + 2] * r[ix[x * 4 + 2]];
        float a3 = wx[x * 4 + 3] * r[ix[x * 4 + 3]];
        acc += wy[y * 4 + m] * ((a0 + a1) + (a2 + a3));
      }
      dst[x] = acc;
    }
  }
}

// src/cpu.rs:960-995
void upsample2x_nearest(const float* in, int c, int h, int w, float* out) {
  int ow = w * 2;
#pragma omp parallel for schedule(static)
  for (int i = 0; i < c * h; i++) {
    const float* src = in + (size_t)i * w;
    float* a = out + (size_t)i * 2 * ow;
    float* b = a + ow;
    for (int x = 0; x < w; x++) {
      float v = src[x];
      a[2 * x] = v;
      a[2 * x + 1] = v;
      b[2 * x] = v;
      b[2 * x + 1] = v;
    }
  }
}

std::string S(const char* fmt, int a, int b = 0) {
  char buf[256];
  snprintf(buf, sizeof buf, fmt, a, b);
  return buf;
}

typedef void (*DumpFn)(const char* name, const float* data, int64_t n, void* user);

int run_forward(const Net& net, int h, int w, const float* input, float* out_img, float* aux_img,
                DumpFn dump, void* user) {
  Plan pl(h, w, net.win, net.c);
  int c = net.c, hw = pl.plane(), tokens = pl.tokens(), hidden = net.mlp * c;
  size_t plane = (size_t)hw * c, tokc = (size_t)tokens * c;
  auto D = [&](const std::string& nm, const float* p, size_t n) {
    if (dump) dump(nm.c_str(), p, (int64_t)n, user);
  };
  auto W = [&](const std::string& k) {
    const float* p = net.w(k);
    if (!p) throw std::string("missing tensor " + k);
    return p;
  };
  std::vector<float> padded = pad_reflect(input, 3, h, w, pl.hp, pl.wp);
  std::vector<float> cur(plane), acc(plane), stage(plane), res(plane);
  conv3x3(padded.data(), 3, pl.hp, pl.wp, W("conv_first.weight"), c, W("conv_first.bias"),
          cur.data());
  std::vector<float> body_res = cur;
  D("conv_first", cur.data(), plane);
  conv1x1(cur.data(), c, hw, W("patch_embed.proj.weight"), c, W("patch_embed.proj.bias"),
          acc.data());
  channel_layer_norm(acc.data(), W("patch_embed.norm.weight"), W("patch_embed.norm.bias"),
                     cur.data(), c, hw);
  D("patch_embed", cur.data(), plane);
  std::vector<float> tok(tokc), tok2(tokc), attn(tokc), qkv(3 * tokc), mlp((size_t)tokens * hidden);
  std::vector<float> zero_bias(c, 0.0f), tmp(plane);
  for (size_t s = 0; s < net.depths.size(); s++) {
    stage = cur;
    res = cur;
    for (int b = 0; b < net.depths[s]; b++) {
      int shift = pl.shift_for(b);
      std::string p = S("layers.%d.residual_group.blocks.%d", (int)s, b);
      gather(pl, cur.data(), shift, tok.data());
      linear(tok.data(), tokens, c, W(p + ".attn.qkv.wq"), c, W(p + ".attn.qkv.q_bias"),
             qkv.data());
      linear(tok.data(), tokens, c, W(p + ".attn.qkv.wk"), c, zero_bias.data(),
             qkv.data() + tokc);
      linear(tok.data(), tokens, c, W(p + ".attn.qkv.wv"), c, W(p + ".attn.qkv.v_bias"),
             qkv.data() + 2 * tokc);
      attention(pl, net.heads, net.hd, W(p + ".attn.logit_scale"), W(p + ".attn.cpb_pre"),
                qkv.data(), shift, attn.data());
      linear(attn.data(), tokens, c, W(p + ".attn.proj.weight"), c, W(p + ".attn.proj.bias"),
             tok2.data());
      scatter(pl, tok2.data(), shift, acc.data());
      channel_layer_norm(acc.data(), W(p + ".norm1.weight"), W(p + ".norm1.bias"), tmp.data(), c,
                         hw);
      add_into(tmp.data(), res.data(), plane);
      gather(pl, res.data(), shift, tok.data());
      linear(tok.data(), tokens, c, W(p + ".mlp.fc1.weight"), hidden, W(p + ".mlp.fc1.bias"),
             mlp.data());
      gelu_erf_inplace(mlp.data(), mlp.size());
      linear(mlp.data(), tokens, hidden, W(p + ".mlp.fc2.weight"), c, W(p + ".mlp.fc2.bias"),
             attn.data());
      scatter(pl, attn.data(), shift, acc.data());
      channel_layer_norm(acc.data(), W(p + ".norm2.weight"), W(p + ".norm2.bias"), tmp.data(), c,
                         hw);
      add_into(tmp.data(), res.data(), plane);
      cur = res;
      D(S("layers.%d.blocks.%d", (int)s, b), cur.data(), plane);
    }
    conv3x3(cur.data(), c, pl.hp, pl.wp, W(S("layers.%d.conv.weight", (int)s)), c,
            W(S("layers.%d.conv.bias", (int)s)), acc.data());
    conv1x1(acc.data(), c, hw, W(S("layers.%d.patch_embed.proj.weight", (int)s)), c,
            W(S("layers.%d.patch_embed.proj.bias", (int)s)), cur.data());
    add_into(stage.data(), cur.data(), plane);
    D(S("layers.%d", (int)s), cur.data(), plane);
  }
  std::vector<float> nbuf(plane);
  channel_layer_norm(cur.data(), W("norm.weight"), W("norm.bias"), nbuf.data(), c, hw);
  D("norm", nbuf.data(), plane);
  conv3x3(nbuf.data(), c, pl.hp, pl.wp, W("conv_after_body.weight"), c, W("conv_after_body.bias"),
          acc.data());
  add_into(body_res.data(), acc.data(), plane);
  cur = acc;
  D("conv_after_body", cur.data(), plane);

  int scale = net.scale;
  std::vector<float> bic;
  if (net.ups == 3) {
    int feat = (int)(net.n.at("conv_bicubic.weight") / (3 * 9));
    int oh = pl.hp * scale, ow = pl.wp * scale;
    std::vector<float> resized((size_t)3 * oh * ow);
    bicubic_resize(padded.data(), 3, pl.hp, pl.wp, oh, ow, resized.data());
    D("bicubic_resize", resized.data(), resized.size());
    bic.resize((size_t)feat * oh * ow);
    conv3x3(resized.data(), 3, oh, ow, W("conv_bicubic.weight"), feat, W("conv_bicubic.bias"),
            bic.data());
    D("conv_bicubic", bic.data(), bic.size());
  }
  // head (src/cpu.rs:1701-1880)
  std::vector<float> planes, aux;
  int h2 = pl.hp, w2 = pl.wp;
  if (net.ups == 0 || net.ups == 3) {
    int feat = (int)(net.n.at("conv_before_upsample.0.weight") / ((int64_t)c * 9));
    std::vector<float> a((size_t)feat * hw);
    conv3x3(cur.data(), c, pl.hp, pl.wp, W("conv_before_upsample.0.weight"), feat,
            W("conv_before_upsample.0.bias"), a.data());
    leaky_relu(a.data(), a.size(), 0.01f);
    D("conv_before_upsample", a.data(), a.size());
    if (net.ups == 3) {
      aux.resize((size_t)3 * hw);
      conv3x3(a.data(), feat, pl.hp, pl.wp, W("conv_aux.weight"), 3, W("conv_aux.bias"),
              aux.data());
      D("conv_aux", aux.data(), aux.size());
      std::vector<float> x((size_t)feat * hw);
      conv3x3(aux.data(), 3, pl.hp, pl.wp, W("conv_after_aux.0.weight"), feat,
              W("conv_after_aux.0.bias"), x.data());
      leaky_relu(x.data(), x.size(), 0.01f);
      a.swap(x);
    }
    int oct = (int)std::lround(std::log2((double)scale));
    for (int o = 0; o < oct; o++) {
      std::vector<float> shuf((size_t)feat * 4 * h2 * w2);
      conv3x3_shuffle2(a.data(), feat, h2, w2, W(S("upsample.%d.weight", 2 * o)), feat,
                       W(S("upsample.%d.bias", 2 * o)), shuf.data());
      a.swap(shuf);
      h2 *= 2;
      w2 *= 2;
      D(S("upsample.%d", o), a.data(), a.size());
    }
    if (net.ups == 3) add_into(bic.data(), a.data(), a.size());
    planes.resize((size_t)3 * h2 * w2);
    conv3x3(a.data(), feat, h2, w2, W("conv_last.weight"), 3, W("conv_last.bias"), planes.data());
  } else if (net.ups == 1) {
    int oc = 3 * scale * scale;
    std::vector<float> up((size_t)oc * hw);
    conv3x3(cur.data(), c, pl.hp, pl.wp, W("upsample.0.weight"), oc, W("upsample.0.bias"),
            up.data());
    h2 = pl.hp * scale;
    w2 = pl.wp * scale;
    planes.resize((size_t)3 * h2 * w2);
    pixel_shuffle(up.data(), 3, pl.hp, pl.wp, scale, planes.data());
  } else {
    int feat = (int)(net.n.at("conv_before_upsample.0.weight") / ((int64_t)c * 9));
    std::vector<float> a((size_t)feat * hw);
    conv3x3(cur.data(), c, pl.hp, pl.wp, W("conv_before_upsample.0.weight"), feat,
            W("conv_before_upsample.0.bias"), a.data());
    leaky_relu(a.data(), a.size(), 0.01f);
    D("conv_before_upsample", a.data(), a.size());
    const char* names[2] = {"conv_up1", "conv_up2"};
    for (int st = 0; st < 2; st++) {
      std::vector<float> up((size_t)feat * 4 * h2 * w2);
      upsample2x_nearest(a.data(), feat, h2, w2, up.data());
      h2 *= 2;
      w2 *= 2;
      std::vector<float> b((size_t)feat * h2 * w2);
      conv3x3(up.data(), feat, h2, w2, W(std::string(names[st]) + ".weight"), feat,
              W(std::string(names[st]) + ".bias"), b.data());
      leaky_relu(b.data(), b.size(), 0.2f);
      a.swap(b);
    }
    std::vector<float> hr((size_t)feat * h2 * w2);
    conv3x3(a.data(), feat, h2, w2, W("conv_hr.weight"), feat, W("conv_hr.bias"), hr.data());
    leaky_relu(hr.data(), hr.size(), 0.2f);
    planes.resize((size_t)3 * h2 * w2);
    conv3x3(hr.data(), feat, h2, w2, W("conv_last.weight"), 3, W("conv_last.bias"), planes.data());
  }
  // finish (src/cpu.rs:1925-1941): denormalise, crop; aux: denormalise, no crop.
  int oh = h * scale, ow = w * scale;
  for (int ci = 0; ci < 3; ci++)
    for (int y = 0; y < oh; y++)
      for (int x = 0; x < ow; x++)
        out_img[((size_t)ci * oh + y) * ow + x] =
            planes[((size_t)ci * h2 + y) * w2 + x] / net.img_range + net.mean[ci];
  if (net.ups == 3 && aux_img) {
    for (int ci = 0; ci < 3; ci++)
      for (int p = 0; p < hw; p++)
        aux_img[(size_t)ci * hw + p] = aux[(size_t)ci * hw + p] / net.img_range + net.mean[ci];
  }
  return 0;
}

}  // namespace

extern "C" {

typedef struct {
  const char* name;
  const float* data;
  int64_t numel;
} oracle_tensor;

typedef struct {
  int upsampler;  // 0 pixelshuffle, 1 pixelshuffledirect, 2 nearest+conv, 3 pixelshuffle_aux
  int scale, window, embed, heads, mlp_ratio, n_depths;
  int depths[16];
  float img_range;
  float mean[3];
} oracle_config;

void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#endif
  (void)n;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

// One whole forward: input [3][h][w] mean-adjusted, output [3][h*s][w*s], aux [3][hp][wp].
int oracle_forward(const oracle_config* cfg, const oracle_tensor* ts, int nt, int h, int w,
                   const float* input, float* out, float* aux, DumpFn dump, void* user) {
  Net net;
  net.ups = cfg->upsampler;
  net.scale = cfg->scale;
  net.win = cfg->window;
  net.c = cfg->embed;
  net.heads = cfg->heads;
  net.hd = cfg->embed / cfg->heads;
  net.mlp = cfg->mlp_ratio;
  net.depths.assign(cfg->depths, cfg->depths + cfg->n_depths);
  net.img_range = cfg->img_range;
  for (int i = 0; i < 3; i++) net.mean[i] = cfg->mean[i];
  for (int i = 0; i < nt; i++) {
    net.t[ts[i].name] = ts[i].data;
    net.n[ts[i].name] = ts[i].numel;
  }
  try {
    return run_forward(net, h, w, input, out, aux, dump, user);
  } catch (const std::string& e) {
    (void)e;
    return -1;
  }
}

void oracle_bicubic(const float* in, int c, int h, int w, int oh, int ow, float* out) {
  bicubic_resize(in, c, h, w, oh, ow, out);
}

void oracle_conv3x3(const float* in, int ci, int h, int w, const float* wgt, int co,
                    const float* bias, float* out) {
  conv3x3(in, ci, h, w, wgt, co, bias, out);
}

void oracle_linear(const float* x, int rows, int ci, const float* wgt, int co, const float* bias,
                   float* out) {
  linear(x, rows, ci, wgt, co, bias, out);
}

void oracle_layer_norm(const float* x, const float* w, const float* b, float* y, int c, int hw) {
  channel_layer_norm(x, w, b, y, c, hw);
}

// Window attention on a plane: qkv [3][tokens][c] (window-major tokens), out [tokens][c].
void oracle_attention(int h, int w, int win, int c, int heads, const float* logit_scale,
                      const float* cpb, const float* qkv, int shift, float* out) {
  Plan pl(h, w, win, c);
  // h, w are the PADDED plane here: rebuild a plan whose hp/wp equal them.
  pl.hp = h;
  pl.wp = w;
  pl.nwh = h / win;
  pl.nww = w / win;
  pl.nw = pl.nwh * pl.nww;
  attention(pl, heads, c / heads, logit_scale, cpb, qkv, shift, out);
}

float oracle_fast_exp(float x) { return fast_exp(x); }

void oracle_pad_reflect(const float* x, int c, int h, int w, int hp, int wp, float* out) {
  std::vector<float> o = pad_reflect(x, c, h, w, hp, wp);
  memcpy(out, o.data(), sizeof(float) * o.size());
}

}  // extern "C"
