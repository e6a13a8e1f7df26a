// CPU restatement of the subset of AMD's aie_api (MLIR-AIE v1.3.4, not present
// here) that the reference's row kernels use, so that their own sources
// (kernels/gelu_row4*.cc, softmax_row*.cc, layer_norm_gb.cc) compile with g++
// and run on the host as a test oracle. TEST INFRASTRUCTURE ONLY.
//
// Semantics restated (the AIE2 vector unit):
//   * bfloat16 vectors hold bf16 values; arithmetic producing a bf16 vector is
//     done in fp32 and converted with the current rounding mode.
//   * accum<accfloat> holds fp32; bf16 x bf16 products are exact in fp32, and
//     accumulator adds round to nearest even.
//   * the rounding mode is global state: truncation toward zero by default,
//     round-to-nearest-even after set_rounding(conv_even). Scalar
//     float -> bfloat16 casts use the same mode.
//   * reduce_add folds lanes with a halving tree (l with l+N/2, ...), the
//     order the build's oracle and CUDA kernels also use.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

namespace aie_shim {
// Internal linkage: every kernel library built from this header has its own
// mode, starting at truncation, as each AIE core running one kernel does.
static int g_mode = 0;  // 0 = truncate toward zero, 1 = round to nearest even
inline int &rounding() { return g_mode; }
inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint16_t to_bf16_bits(float f) {
  uint32_t u = f2u(f);
  if (std::isnan(f)) return (uint16_t)((u >> 16) | 0x40);
  if (rounding() == 0) return (uint16_t)(u >> 16);
  uint32_t bias = ((u >> 16) & 1u) + 0x7FFFu;
  return (uint16_t)((uint64_t(u) + bias) >> 16);
}
}  // namespace aie_shim

struct bfloat16 {
  uint16_t bits;
  bfloat16() : bits(0) {}
  bfloat16(float f) : bits(aie_shim::to_bf16_bits(f)) {}
  operator float() const { return aie_shim::u2f(uint32_t(bits) << 16); }
};

struct accfloat {};

namespace aie {

enum class rounding_mode { floor = 0, conv_even = 1 };
inline void set_rounding(rounding_mode m) {
  aie_shim::rounding() = (m == rounding_mode::conv_even) ? 1 : 0;
}

template <typename T, int N> struct vector {
  T v[N];
  T &operator[](int i) { return v[i]; }
  const T &operator[](int i) const { return v[i]; }
};

template <int N> struct mask {
  bool m[N];
};

template <typename A, int N> struct accum;

template <int N> struct accum<accfloat, N> {
  float v[N];
  accum() { for (int i = 0; i < N; i++) v[i] = 0.f; }
  template <typename T> vector<T, N> to_vector() const {
    vector<T, N> r;
    for (int i = 0; i < N; i++) r.v[i] = T(v[i]);
    return r;
  }
  void from_vector(const vector<float, N> &x) {
    for (int i = 0; i < N; i++) v[i] = x.v[i];
  }
  operator vector<float, N>() const { return to_vector<float>(); }
  operator vector<bfloat16, N>() const { return to_vector<bfloat16>(); }
};

template <typename T, int N> vector<T, N> broadcast(T x) {
  vector<T, N> r;
  for (int i = 0; i < N; i++) r.v[i] = x;
  return r;
}

template <typename T, int N> vector<T, N> zeros_v() {
  vector<T, N> r;
  for (int i = 0; i < N; i++) r.v[i] = T(0.f);
  return r;
}

template <typename T, int N> struct zeros_helper {
  static vector<T, N> get() { return zeros_v<T, N>(); }
};
template <int N> struct zeros_helper<accfloat, N> {
  static accum<accfloat, N> get() { return accum<accfloat, N>(); }
};
template <typename T, int N> auto zeros() { return zeros_helper<T, N>::get(); }

// bf16 vector arithmetic: fp32 result converted with the rounding mode
template <int N>
vector<bfloat16, N> sub(const vector<bfloat16, N> &a, const vector<bfloat16, N> &b) {
  vector<bfloat16, N> r;
  for (int i = 0; i < N; i++) r.v[i] = bfloat16(float(a.v[i]) - float(b.v[i]));
  return r;
}
template <int N>
vector<bfloat16, N> add(const vector<bfloat16, N> &a, const vector<bfloat16, N> &b) {
  vector<bfloat16, N> r;
  for (int i = 0; i < N; i++) r.v[i] = bfloat16(float(a.v[i]) + float(b.v[i]));
  return r;
}
template <int N>
vector<bfloat16, N> max(const vector<bfloat16, N> &a, const vector<bfloat16, N> &b) {
  vector<bfloat16, N> r;
  for (int i = 0; i < N; i++) r.v[i] = float(a.v[i]) >= float(b.v[i]) ? a.v[i] : b.v[i];
  return r;
}
template <int N>
mask<N> lt(const vector<bfloat16, N> &a, const vector<bfloat16, N> &b) {
  mask<N> r;
  for (int i = 0; i < N; i++) r.m[i] = float(a.v[i]) < float(b.v[i]);
  return r;
}
template <int N>
vector<bfloat16, N> select(const vector<bfloat16, N> &a, const vector<bfloat16, N> &b,
                           const mask<N> &m) {
  vector<bfloat16, N> r;
  for (int i = 0; i < N; i++) r.v[i] = m.m[i] ? b.v[i] : a.v[i];
  return r;
}

// products into the fp32 accumulator (bf16 x bf16 is exact in fp32)
template <int N>
accum<accfloat, N> mul(const vector<bfloat16, N> &a, const vector<bfloat16, N> &b) {
  accum<accfloat, N> r;
  for (int i = 0; i < N; i++) r.v[i] = float(a.v[i]) * float(b.v[i]);
  return r;
}
template <int N>
accum<accfloat, N> mul(const vector<bfloat16, N> &a, bfloat16 b) {
  accum<accfloat, N> r;
  for (int i = 0; i < N; i++) r.v[i] = float(a.v[i]) * float(b);
  return r;
}
template <int N>
accum<accfloat, N> mac(const accum<accfloat, N> &acc, const vector<bfloat16, N> &a,
                       const vector<bfloat16, N> &b) {
  accum<accfloat, N> r;
  for (int i = 0; i < N; i++) r.v[i] = acc.v[i] + float(a.v[i]) * float(b.v[i]);
  return r;
}
template <int N>
accum<accfloat, N> add(const accum<accfloat, N> &a, const accum<accfloat, N> &b) {
  accum<accfloat, N> r;
  for (int i = 0; i < N; i++) r.v[i] = a.v[i] + b.v[i];
  return r;
}
template <int N>
accum<accfloat, N> add(const accum<accfloat, N> &a, const vector<bfloat16, N> &b) {
  accum<accfloat, N> r;
  for (int i = 0; i < N; i++) r.v[i] = a.v[i] + float(b.v[i]);
  return r;
}
template <int N>
accum<accfloat, N> sub(const accum<accfloat, N> &a, const accum<accfloat, N> &b) {
  accum<accfloat, N> r;
  for (int i = 0; i < N; i++) r.v[i] = a.v[i] - b.v[i];
  return r;
}

// fp32 vectors (layer_norm_gb.cc)
template <int N>
vector<float, N> add(const vector<float, N> &a, const vector<float, N> &b) {
  vector<float, N> r;
  for (int i = 0; i < N; i++) r.v[i] = a.v[i] + b.v[i];
  return r;
}

template <int N> float reduce_add(vector<float, N> x) {
  for (int h = N / 2; h >= 1; h /= 2)
    for (int i = 0; i < h; i++) x.v[i] = x.v[i] + x.v[i + h];
  return x.v[0];
}
template <int N> bfloat16 reduce_max(const vector<bfloat16, N> &x) {
  bfloat16 m = x.v[0];
  for (int i = 1; i < N; i++)
    if (float(x.v[i]) > float(m)) m = x.v[i];
  return m;
}

inline float inv(float x) { return 1.0f / x; }

// iterators over memory, one N-wide vector per step: cbegin_* read,
// begin_* write
template <typename T, int N> struct read_it {
  const T *p;
  vector<T, N> operator*() const {
    vector<T, N> r;
    std::memcpy(r.v, p, sizeof(T) * N);
    return r;
  }
  read_it operator++(int) { read_it old = *this; p += N; return old; }
};
template <typename T, int N> struct write_it {
  T *p;
  struct proxy {
    T *p;
    proxy &operator=(const vector<T, N> &x) {
      std::memcpy(p, x.v, sizeof(T) * N);
      return *this;
    }
  };
  proxy operator*() const { return proxy{p}; }
  write_it operator++(int) { write_it old = *this; p += N; return old; }
};

template <int N, typename T> read_it<T, N> cbegin_vector(T *p) { return {p}; }
template <int N, typename T> read_it<T, N> cbegin_restrict_vector(T *p) { return {p}; }
template <int N, typename T> write_it<T, N> begin_vector(T *p) { return {p}; }
template <int N, typename T> write_it<T, N> begin_restrict_vector(T *p) { return {p}; }

template <int N, typename T> vector<T, N> load_v(const T *p) {
  vector<T, N> r;
  std::memcpy(r.v, p, sizeof(T) * N);
  return r;
}
template <typename T, int N> void store_v(T *p, const vector<T, N> &x) {
  std::memcpy(p, x.v, sizeof(T) * N);
}

}  // namespace aie

// helper used by the softmax kernels (MLIR-AIE aie_kernels)
inline aie::vector<bfloat16, 16> to_v16bfloat16(const aie::accum<accfloat, 16> &a) {
  return a.to_vector<bfloat16>();
}
