// resize.cuh — camera-frame resize with padding (the reference's resize_with_pad,
// docs/archive/windows/π05_네이티브엔진.md:296-297, after openpi image_tools.resize_with_pad over Pillow's
// 8-bit bilinear filter), shared by the host function pi05_resize_with_pad and the device kernel that
// pi05_act_batch runs on camera frames.
//
// Geometry (openpi): ratio = max(w / out_w, h / out_h) in double precision; the resized image is
// int(w / ratio) x int(h / ratio), pasted at (int((out_w - rw) / 2), int((out_h - rh) / 2)) into a
// zero frame; a frame already of the output size is copied unchanged.
//
// Resampling (Pillow's 8-bit bilinear "reduce-aware" filter, restated): separable, one pass per axis
// whose size changes (width first, then height).  Output sample i of an axis of n_in -> n_out samples
// has centre c = (i + 0.5) * s, s = n_in / n_out; the triangle filter is widened by f = max(s, 1)
// (support f), taps x in [int(c - f + 0.5) clamped at 0, int(c + f + 0.5) clamped at n_in), weights
// tri((x - c + 0.5) / f) normalised to sum 1, then rounded to fixed point with 22 fraction bits
// (round half away from zero).  A pass accumulates the 8-bit samples times the integer weights from
// 2^21 (rounding), shifts by 22 and clamps to [0, 255].  The tap tables are built on the host in
// double precision; the device kernel reads them, so both paths do the same integer arithmetic.
#pragma once
#include <cmath>
#include <cstdint>
#include <vector>

namespace p5rs {

constexpr int RS_BITS = 22;

// Tap table of one axis: per output sample its first input sample, its tap count and `taps` weights.
struct AxisTaps {
  int taps = 0;
  std::vector<int> first, count;
  std::vector<int32_t> w;  // [n_out][taps]
};

inline AxisTaps axis_taps(int n_in, int n_out) {
  AxisTaps t;
  const double s = (double)n_in / (double)n_out;
  const double f = s < 1.0 ? 1.0 : s;
  t.taps = (int)std::ceil(f) * 2 + 1;
  t.first.resize(n_out);
  t.count.resize(n_out);
  t.w.assign((size_t)n_out * t.taps, 0);
  std::vector<double> k(t.taps);
  for (int i = 0; i < n_out; ++i) {
    const double c = (i + 0.5) * s;
    int lo = (int)(c - f + 0.5);
    if (lo < 0) lo = 0;
    int hi = (int)(c + f + 0.5);
    if (hi > n_in) hi = n_in;
    const int cnt = hi - lo;
    double sum = 0.0;
    for (int x = 0; x < cnt; ++x) {
      const double d = std::fabs((x + lo - c + 0.5) / f);
      k[x] = d < 1.0 ? 1.0 - d : 0.0;
      sum += k[x];
    }
    for (int x = 0; x < cnt; ++x) {
      const double v = sum != 0.0 ? k[x] / sum : k[x];
      const double q = v * (double)(1 << RS_BITS);
      t.w[(size_t)i * t.taps + x] = (int32_t)(q < 0.0 ? q - 0.5 : q + 0.5);
    }
    t.first[i] = lo;
    t.count[i] = cnt;
  }
  return t;
}

// Resized extent and paste offset of an h x w frame in an out_h x out_w frame; false if degenerate.
struct Geometry {
  int rh, rw, pad_h, pad_w;
};

inline bool geometry(int h, int w, int out_h, int out_w, Geometry* g) {
  if (h == out_h && w == out_w) {
    *g = {h, w, 0, 0};
    return true;
  }
  const double ratio = std::fmax((double)w / (double)out_w, (double)h / (double)out_h);
  const int rh = (int)((double)h / ratio), rw = (int)((double)w / ratio);
  if (rh < 1 || rw < 1 || rh > out_h || rw > out_w) return false;
  const int pad_h = (int)((out_h - rh) / 2.0), pad_w = (int)((out_w - rw) / 2.0);
  *g = {rh, rw, pad_h < 0 ? 0 : pad_h, pad_w < 0 ? 0 : pad_w};
  return true;
}

__host__ __device__ inline uint8_t clip8(int32_t acc) {
  if (acc <= 0) return 0;
  const int32_t v = acc >> RS_BITS;
  return v > 255 ? 255 : (uint8_t)v;
}

// One frame for the device kernel.  Tables (int32, in one device buffer at `tab`): width axis first[rw],
// count[rw], weights[rw][tw]; then height axis first[rh], count[rh], weights[rh][th].  An axis whose size
// does not change (rw == w, rh == h) has no table and no pass.
struct FrameJob {
  const uint8_t* src;
  long stride;
  int h, w, ch;
  int rh, rw, pad_h, pad_w;
  int tw, th;         // taps per output sample (weight row length) of each axis
  long tab_w, tab_h;  // offsets of the two tables in the table buffer (-1: no pass on that axis)
  uint8_t* dst;       // [out_h][out_w][3]
};

}  // namespace p5rs

#if defined(__CUDACC__) && !defined(P5RS_HOST_ONLY)
// One thread per output pixel of one frame (blockIdx.y = frame): the width pass of every input row the
// height pass reads is recomputed in registers, with the same integer arithmetic as the host passes
// (which store the width pass as 8-bit samples first), so the result is bit-identical.
__global__ void resize_with_pad_kernel(const p5rs::FrameJob* jobs, const int32_t* tab, int out_h, int out_w) {
  using namespace p5rs;
  const FrameJob J = jobs[blockIdx.y];
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= out_h * out_w) return;
  const int oy = p / out_w, ox = p % out_w;
  uint8_t* d = J.dst + (size_t)p * 3;
  const int y = oy - J.pad_h, x = ox - J.pad_w;
  if (y < 0 || y >= J.rh || x < 0 || x >= J.rw) {
    d[0] = d[1] = d[2] = 0;
    return;
  }
  const int32_t* wf = J.tab_w >= 0 ? tab + J.tab_w : nullptr;  // width table: first, count, weights
  const int32_t* hf = J.tab_h >= 0 ? tab + J.tab_h : nullptr;
  int x0 = x, nx = 0;
  const int32_t* wx = nullptr;
  if (wf) {
    x0 = wf[x];
    nx = wf[J.rw + x];
    wx = wf + 2 * J.rw + (size_t)x * J.tw;
  }
  auto sample = [&](int row, int c) -> int32_t {  // width-pass value of input row `row`, channel c
    const uint8_t* r = J.src + (size_t)row * J.stride;
    if (!wf) return r[(size_t)x * J.ch + c];
    int32_t acc = 1 << (RS_BITS - 1);
    for (int i = 0; i < nx; ++i) acc += (int32_t)r[(size_t)(x0 + i) * J.ch + c] * wx[i];
    return clip8(acc);
  };
  for (int c = 0; c < 3; ++c) {
    int32_t v;
    if (hf) {
      const int y0 = hf[y], ny = hf[J.rh + y];
      const int32_t* wy = hf + 2 * J.rh + (size_t)y * J.th;
      int32_t acc = 1 << (RS_BITS - 1);
      for (int j = 0; j < ny; ++j) acc += sample(y0 + j, c) * wy[j];
      v = clip8(acc);
    } else {
      v = sample(y, c);
    }
    d[c] = (uint8_t)v;
  }
}
#endif
