// preprocess.cu — host-side camera-frame preprocessing (the reference's resize_with_pad,
// π05_네이티브엔진.md:296-297, after openpi's image_tools.resize_with_pad over Pillow's bilinear resize;
// geometry and filter in resize.cuh, shared with the device kernel of pi05_act_batch) and the state /
// action transforms of the reference wrapper.  Host code only; no GPU is involved.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/pi05.h"
#define P5RS_HOST_ONLY  // the device kernel is compiled with the engine
#include "resize.cuh"

namespace {

using p5rs::AxisTaps;
using p5rs::axis_taps;
using p5rs::RS_BITS;
inline uint8_t rs_clip(int32_t acc) { return p5rs::clip8(acc); }

// width pass: in [h][w_in][3] -> out [h][w_out][3]
void resample_width(const uint8_t* in, int h, int w_in, uint8_t* out, int w_out) {
  const AxisTaps t = axis_taps(w_in, w_out);
  for (int y = 0; y < h; ++y) {
    const uint8_t* row = in + (size_t)y * w_in * 3;
    uint8_t* orow = out + (size_t)y * w_out * 3;
    for (int i = 0; i < w_out; ++i) {
      const int32_t* wi = &t.w[(size_t)i * t.taps];
      for (int ch = 0; ch < 3; ++ch) {
        int32_t acc = 1 << (RS_BITS - 1);
        for (int x = 0; x < t.count[i]; ++x) acc += (int32_t)row[(size_t)(t.first[i] + x) * 3 + ch] * wi[x];
        orow[(size_t)i * 3 + ch] = rs_clip(acc);
      }
    }
  }
}

// height pass: in [h_in][w][3] -> out [h_out][w][3]
void resample_height(const uint8_t* in, int h_in, int w, uint8_t* out, int h_out) {
  const AxisTaps t = axis_taps(h_in, h_out);
  for (int i = 0; i < h_out; ++i) {
    const int32_t* wi = &t.w[(size_t)i * t.taps];
    uint8_t* orow = out + (size_t)i * w * 3;
    for (int e = 0; e < w * 3; ++e) {
      int32_t acc = 1 << (RS_BITS - 1);
      for (int y = 0; y < t.count[i]; ++y) acc += (int32_t)in[(size_t)(t.first[i] + y) * w * 3 + e] * wi[y];
      orow[e] = rs_clip(acc);
    }
  }
}

}  // namespace

extern "C" {

int pi05_resize_with_pad(const uint8_t* src, int h, int w, int channels, long stride, uint8_t* dst, int out_h,
                         int out_w) {
  if (!src || !dst || h < 1 || w < 1 || out_h < 1 || out_w < 1 || (channels != 3 && channels != 4) ||
      stride < (long)w * channels)
    return PI05_ERR_ARG;
  // RGB rows, contiguous (alpha dropped)
  std::vector<uint8_t> rgb((size_t)h * w * 3);
  for (int y = 0; y < h; ++y)
    for (int x = 0; x < w; ++x)
      memcpy(&rgb[((size_t)y * w + x) * 3], src + (size_t)y * stride + (size_t)x * channels, 3);
  if (h == out_h && w == out_w) {
    memcpy(dst, rgb.data(), rgb.size());
    return PI05_OK;
  }
  p5rs::Geometry geo;
  if (!p5rs::geometry(h, w, out_h, out_w, &geo)) return PI05_ERR_ARG;
  const int rh = geo.rh, rw = geo.rw;
  std::vector<uint8_t> a = rgb, b;
  int ch = h, cw = w;
  if (rw != cw) {
    b.resize((size_t)ch * rw * 3);
    resample_width(a.data(), ch, cw, b.data(), rw);
    a.swap(b);
    cw = rw;
  }
  if (rh != ch) {
    b.resize((size_t)rh * cw * 3);
    resample_height(a.data(), ch, cw, b.data(), rh);
    a.swap(b);
    ch = rh;
  }
  const int pad_h = geo.pad_h, pad_w = geo.pad_w;
  memset(dst, 0, (size_t)out_h * out_w * 3);
  for (int y = 0; y < rh; ++y)
    memcpy(dst + ((size_t)(y + pad_h) * out_w + pad_w) * 3, &a[(size_t)y * rw * 3], (size_t)rw * 3);
  return PI05_OK;
}

// openpi Normalize / Unnormalize in float32, per dimension j of x[n][dim], in place:
//   mode 0 (z-score, a = mean, b = std):   y = (x - a) / (b + 1e-6)        inverse x = y * (b + 1e-6) + a
//   mode 1 (quantile, a = q01, b = q99):   y = (x - a) / (b - a + 1e-6) * 2 - 1
//                                          inverse x = (y + 1) / 2 * (b - a + 1e-6) + a
int pi05_normalize(float* x, int n, int dim, const float* a, const float* b, int mode, int inverse) {
  if (!x || !a || !b || n < 0 || dim < 1 || (mode != 0 && mode != 1)) return PI05_ERR_ARG;
  const float eps = 1e-6f;
  for (long i = 0; i < (long)n * dim; ++i) {
    const int j = (int)(i % dim);
    const float v = x[i];
    if (mode == 0)
      x[i] = inverse ? v * (b[j] + eps) + a[j] : (v - a[j]) / (b[j] + eps);
    else
      x[i] = inverse ? (v + 1.0f) / 2.0f * (b[j] - a[j] + eps) + a[j] : (v - a[j]) / (b[j] - a[j] + eps) * 2.0f - 1.0f;
  }
  return PI05_OK;
}

// State discretisation of the pi0.5 prompt (openpi): bin = (number of edges <= x) - 1 over the `bins`
// edges -1 + 2k / bins, k = 0 .. bins-1 (numpy digitize of linspace(-1, 1, bins + 1)[:-1], minus one):
// -1 below -1, bins - 1 at or above 1 - 2 / bins.  The edges are exact in binary for power-of-two bins.
// NaN lands in bin bins - 1, as numpy's digitize sorts NaN after every edge.
int pi05_discretize_state(const float* x, int n, int dim, int bins, int32_t* out) {
  if (!x || !out || n < 0 || dim < 1 || bins < 1) return PI05_ERR_ARG;
  for (long i = 0; i < (long)n * dim; ++i) {
    const double v = x[i];
    if (std::isnan(v)) {
      out[i] = bins - 1;
      continue;
    }
    int lo = 0, hi = bins;  // count of edges <= v, by bisection over the increasing edges
    while (lo < hi) {
      const int mid = (lo + hi) / 2;
      if (-1.0 + 2.0 * mid / bins <= v)
        lo = mid + 1;
      else
        hi = mid;
    }
    out[i] = lo - 1;
  }
  return PI05_OK;
}

// Delta to absolute actions (openpi AbsoluteActions): actions[t][j] += state[j] for the dimensions j
// with mask[j] != 0, t < horizon, in place.
int pi05_absolute_actions(float* actions, int horizon, int dim, const float* state, const uint8_t* mask) {
  if (!actions || !state || !mask || horizon < 0 || dim < 1) return PI05_ERR_ARG;
  for (int t = 0; t < horizon; ++t)
    for (int j = 0; j < dim; ++j)
      if (mask[j]) actions[(size_t)t * dim + j] += state[j];
  return PI05_OK;
}

// Cubic resampling of an executed action segment (the PiBehavior wrapper replays 26 actions in 20 steps,
// π05_네이티브엔진.md:143 and :146; there scipy interp1d(kind="cubic")): per dimension, the not-a-knot cubic spline
// through (i, in[i][j]), i = 0..n_in-1, evaluated at x_k = k (n_in - 1) / (n_out - 1).  The spline's second
// derivatives M solve, with unit knot spacing, M[i-1] + 4 M[i] + M[i+1] = 6 (y[i-1] - 2 y[i] + y[i+1]) inside
// and M[0] - 2 M[1] + M[2] = 0, M[n-3] - 2 M[n-2] + M[n-1] = 0 (a continuous third derivative at the
// second and the second-to-last knot); the system is solved in double precision by Gaussian elimination
// with partial pivoting.
int pi05_interp_actions_cubic(const float* in, int n_in, int dim, float* out, int n_out) {
  if (!in || !out || n_in < 4 || n_in > 4096 || dim < 1 || n_out < 2) return PI05_ERR_ARG;
  const int n = n_in;
  std::vector<double> A((size_t)n * n), M(n), y(n);
  std::vector<int> piv(n);
  for (int j = 0; j < dim; ++j) {
    for (int i = 0; i < n; ++i) y[i] = in[(size_t)i * dim + j];
    std::fill(A.begin(), A.end(), 0.0);
    A[0] = 1.0, A[1] = -2.0, A[2] = 1.0, M[0] = 0.0;
    for (int i = 1; i < n - 1; ++i) {
      A[(size_t)i * n + i - 1] = 1.0, A[(size_t)i * n + i] = 4.0, A[(size_t)i * n + i + 1] = 1.0;
      M[i] = 6.0 * (y[i - 1] - 2.0 * y[i] + y[i + 1]);
    }
    A[(size_t)(n - 1) * n + n - 3] = 1.0, A[(size_t)(n - 1) * n + n - 2] = -2.0, A[(size_t)(n - 1) * n + n - 1] = 1.0;
    M[n - 1] = 0.0;
    for (int c = 0; c < n; ++c) {  // forward elimination
      int p = c;
      for (int r = c + 1; r < n; ++r)
        if (std::fabs(A[(size_t)r * n + c]) > std::fabs(A[(size_t)p * n + c])) p = r;
      if (p != c) {
        for (int k = 0; k < n; ++k) std::swap(A[(size_t)c * n + k], A[(size_t)p * n + k]);
        std::swap(M[c], M[p]);
      }
      for (int r = c + 1; r < n; ++r) {
        const double f = A[(size_t)r * n + c] / A[(size_t)c * n + c];
        if (f == 0.0) continue;
        for (int k = c; k < n; ++k) A[(size_t)r * n + k] -= f * A[(size_t)c * n + k];
        M[r] -= f * M[c];
      }
    }
    for (int c = n - 1; c >= 0; --c) {  // back substitution
      double v = M[c];
      for (int k = c + 1; k < n; ++k) v -= A[(size_t)c * n + k] * M[k];
      M[c] = v / A[(size_t)c * n + c];
    }
    for (int k = 0; k < n_out; ++k) {
      const double x = (double)k * (n - 1) / (n_out - 1);
      const int i = std::min(n - 2, (int)x);
      const double t = x - i;
      const double b = y[i + 1] - y[i] - (2.0 * M[i] + M[i + 1]) / 6.0;
      out[(size_t)k * dim + j] = (float)(y[i] + t * (b + t * (M[i] / 2.0 + t * (M[i + 1] - M[i]) / 6.0)));
    }
  }
  return PI05_OK;
}

// Stage vote of the PiBehavior wrapper ("2 of the last 3", π05_네이티브엔진.md:143): `recent` holds the
// last n stage predictions, oldest first; the stage predicted at least twice among the last three is the
// new stage, otherwise `current` stays.  max_stage > 0 caps the result (the per-task stage count).
int pi05_stage_vote(const int32_t* recent, int n, int current, int max_stage) {
  if ((!recent && n > 0) || n < 0) return PI05_ERR_ARG;
  int vote = current;
  const int k = std::min(n, 3);
  const int32_t* last = recent + (n - k);
  for (int a = 0; a < k; ++a) {
    int same = 0;
    for (int b2 = 0; b2 < k; ++b2) same += last[b2] == last[a];
    if (same >= 2) {
      vote = last[a];
      break;
    }
  }
  if (max_stage > 0) vote = std::min(vote, max_stage - 1);
  return std::max(vote, 0);
}

}  // extern "C"
