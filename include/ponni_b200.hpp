// ponni_b200.hpp -- C++ drop-in for PONNI's template inference API, over the
// libponni_b200 C ABI (ponni_b200.h).
//
// Mirrors the names and argument meaning of the reference's template mode:
//   layers            src/layers/ponni_*.h        (Matvec<real>(W[in,out]), Bias<real>(b), Relu<real>(n), ...,
//                                                  Save_State<I,real>(n), Binop_Add<I,real>(n), ...)
//   factories         src/ponni_create_model.h    (create_inference_model, _single/_double/_half/_bhalf_precision)
//   Inference         src/ponni_Inference.h       (validate, forward_batch_parallel, save_weights, load_weights,
//                                                  get/set_trainable_parameters, reallocate_internal_state,
//                                                  internal_state_capacity, weight_schema_fingerprint, print)
// Kokkos Views become ponni::View (host, LayoutRight, owning) for parameters
// and host batches, or raw device pointers with a row stride for
// device-resident batches.  Where the reference calls Kokkos::abort this
// throws ponni::Error (status + the reference's message).
#pragma once

#include <cstdint>
#include <cstring>
#include <iostream>
#include <memory>
#include <stdexcept>
#include <string>
#include <tuple>
#include <type_traits>
#include <vector>

#include "ponni_b200.h"

namespace ponni {

struct Error : std::runtime_error {
  ponni_b200_status status;
  Error(ponni_b200_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

// 16-bit storage types (Kokkos::Experimental::half_t / bhalf_t stand-ins).
struct half_t {
  uint16_t bits = 0;
  half_t() = default;
  half_t(float f) : bits(from_float(f)) {}
  operator float() const { return to_float(bits); }
  static uint16_t from_float(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
      if (ax < 0x33000000u) return (uint16_t)sign;
      uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u, sh = 126u - e;
      uint32_t r = m >> sh, rem = m & ((1u << sh) - 1u), hw = 1u << (sh - 1u);
      if (rem > hw || (rem == hw && (r & 1u))) r++;
      return (uint16_t)(sign | r);
    }
    uint32_t r = (((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13), rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
  }
  static float to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu, x;
    if (e == 0) {
      float v = (float)m * 5.9604644775390625e-08f;
      std::memcpy(&x, &v, 4);
      x |= sign;
    } else if (e == 31) {
      x = sign | 0x7f800000u | (m << 13);
    } else {
      x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
  }
};

struct bhalf_t {
  uint16_t bits = 0;
  bhalf_t() = default;
  bhalf_t(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) bits = (uint16_t)((x >> 16) | 0x40u);
    else bits = (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
  }
  operator float() const {
    uint32_t x = (uint32_t)bits << 16;
    float f;
    std::memcpy(&f, &x, 4);
    return f;
  }
};

template <class T> struct dtype_of;
template <> struct dtype_of<float> { static constexpr ponni_b200_dtype value = PONNI_B200_F32; };
template <> struct dtype_of<double> { static constexpr ponni_b200_dtype value = PONNI_B200_F64; };
template <> struct dtype_of<half_t> { static constexpr ponni_b200_dtype value = PONNI_B200_F16; };
template <> struct dtype_of<bhalf_t> { static constexpr ponni_b200_dtype value = PONNI_B200_BF16; };

// Host LayoutRight View of rank 1 or 2 (owning).
template <class T>
struct View {
  std::vector<T> data_;
  size_t e0 = 0, e1 = 1;
  int rank = 0;
  View() = default;
  View(std::string const&, size_t n0) : data_(n0), e0(n0), e1(1), rank(1) {}
  View(std::string const&, size_t n0, size_t n1) : data_(n0 * n1), e0(n0), e1(n1), rank(2) {}
  size_t extent(int i) const { return i == 0 ? e0 : (i == 1 ? e1 : 1); }
  size_t size() const { return data_.size(); }
  bool is_allocated() const { return !data_.empty(); }
  T* data() { return data_.data(); }
  T const* data() const { return data_.data(); }
  T& operator()(size_t i) { return data_[i]; }
  T const& operator()(size_t i) const { return data_[i]; }
  T& operator()(size_t i, size_t j) { return data_[i * e1 + j]; }
  T const& operator()(size_t i, size_t j) const { return data_[i * e1 + j]; }
};

template <class T> inline void deep_copy(View<T>& v, T value) { for (auto& x : v.data_) x = value; }

namespace detail {
struct LayerBase {
  ponni_b200_layer_desc d{};
  std::vector<double> params;  // canonical order, converted to the model dtype at creation
  LayerBase(int kind, int nin, int nout) {
    d.kind = kind;
    d.num_inputs = nin;
    d.num_outputs = nout;
    d.save_index = -1;
  }
};
template <class V> std::vector<double> flat(V const& v) {
  std::vector<double> r(v.size());
  for (size_t i = 0; i < v.size(); ++i) r[i] = (double)(float)v.data_[i];
  return r;
}
template <> inline std::vector<double> flat(View<double> const& v) { return v.data_; }
}  // namespace detail

// ---- layers (src/layers/*.h) ----
template <class real = float, int = 1, int = 1>
struct Matvec : detail::LayerBase {
  Matvec(View<real> const& w, bool trainable = true) : LayerBase(PONNI_B200_MATVEC, (int)w.extent(0), (int)w.extent(1)) {
    params = detail::flat(w);
    if (trainable) d.flags |= PONNI_B200_FLAG_TRAINABLE;
  }
};
template <class real = float, int = 1>
struct Bias : detail::LayerBase {
  Bias(View<real> const& b, bool trainable = true) : LayerBase(PONNI_B200_BIAS, (int)b.extent(0), (int)b.extent(0)) {
    params = detail::flat(b);
    if (trainable) d.flags |= PONNI_B200_FLAG_TRAINABLE;
  }
};
#define PONNI_B200_ACT(NAME, KIND)                                                   \
  template <class real = float, int = 1>                                             \
  struct NAME : detail::LayerBase {                                                  \
    explicit NAME(int n) : LayerBase(KIND, n, n) {}                                  \
  };
PONNI_B200_ACT(Relu, PONNI_B200_RELU)
PONNI_B200_ACT(Selu, PONNI_B200_SELU)
PONNI_B200_ACT(Silu, PONNI_B200_SILU)
PONNI_B200_ACT(Sigmoid, PONNI_B200_SIGMOID)
PONNI_B200_ACT(Tanh, PONNI_B200_TANH)
PONNI_B200_ACT(HardSwish, PONNI_B200_HARD_SWISH)
PONNI_B200_ACT(Mish, PONNI_B200_MISH)
PONNI_B200_ACT(Softmax, PONNI_B200_SOFTMAX)
PONNI_B200_ACT(LogSoftmax, PONNI_B200_LOG_SOFTMAX)
#undef PONNI_B200_ACT
template <class real = float, int = 1>
struct LeakyRelu : detail::LayerBase {
  LeakyRelu(int n, double slope = 0.01) : LayerBase(PONNI_B200_LEAKY_RELU, n, n) { d.scalar[0] = slope; }
};
template <class real = float, int = 1>
struct Elu : detail::LayerBase {
  Elu(int n, double alpha = 1.0) : LayerBase(PONNI_B200_ELU, n, n) { d.scalar[0] = alpha; }
};
template <class real = float, int = 1>
struct Gelu : detail::LayerBase {
  Gelu(int n, bool approximate = false) : LayerBase(PONNI_B200_GELU, n, n) {
    if (approximate) d.flags |= PONNI_B200_FLAG_APPROXIMATE;
  }
};
template <class real = float, int = 1>
struct Softplus : detail::LayerBase {
  Softplus(int n, double beta = 1.0) : LayerBase(PONNI_B200_SOFTPLUS, n, n) { d.scalar[0] = beta; }
};
template <class real = float, int = 1>
struct HardSigmoid : detail::LayerBase {
  HardSigmoid(int n, double alpha = 0.2, double beta = 0.5) : LayerBase(PONNI_B200_HARD_SIGMOID, n, n) {
    d.scalar[0] = alpha;
    d.scalar[1] = beta;
  }
};
template <class real = float, int = 1>
struct MinMaxNorm : detail::LayerBase {
  MinMaxNorm(int n, double out_min = 0.0, double out_max = 1.0, double eps = 1e-12)
      : LayerBase(PONNI_B200_MIN_MAX_NORM, n, n) {
    d.scalar[0] = out_min;
    d.scalar[1] = out_max;
    d.scalar[2] = eps;
  }
};
template <class real = float, int = 1>
struct LayerNorm : detail::LayerBase {
  LayerNorm(int n, double eps = 1e-5, bool trainable = true) : LayerBase(PONNI_B200_LAYER_NORM, n, n) {
    params.assign(2 * (size_t)n, 0.0);
    for (int i = 0; i < n; ++i) params[i] = 1.0;
    d.scalar[0] = eps;
    if (trainable) d.flags |= PONNI_B200_FLAG_TRAINABLE;
  }
  LayerNorm(View<real> const& gamma, View<real> const& beta, double eps = 1e-5, bool trainable = true)
      : LayerBase(PONNI_B200_LAYER_NORM, (int)gamma.extent(0), (int)gamma.extent(0)) {
    if (gamma.extent(0) != beta.extent(0)) throw Error(PONNI_B200_ERR_VALIDATION, "ERROR: LayerNorm gamma and beta size mismatch");
    params = detail::flat(gamma);
    auto b = detail::flat(beta);
    params.insert(params.end(), b.begin(), b.end());
    d.scalar[0] = eps;
    if (trainable) d.flags |= PONNI_B200_FLAG_TRAINABLE;
  }
};
template <int ISAVE, class real = float, int = 1>
struct Save_State : detail::LayerBase {
  explicit Save_State(int n) : LayerBase(PONNI_B200_SAVE_STATE, n, n) { d.save_index = ISAVE; }
};
template <int ISAVE, class real = float, int = 1>
struct Binop_Add : detail::LayerBase {
  explicit Binop_Add(int n) : LayerBase(PONNI_B200_BINOP_ADD, n, n) { d.save_index = ISAVE; }
};
template <int ISAVE, class real = float, int = 1, int = 1>
struct Binop_Concatenate : detail::LayerBase {
  Binop_Concatenate(int nin, int nout, bool after = true) : LayerBase(PONNI_B200_BINOP_CONCATENATE, nin, nout) {
    d.save_index = ISAVE;
    if (after) d.flags |= PONNI_B200_FLAG_AFTER;
  }
};
template <int ISAVE, class real = float, int = 1, int = 1>
struct Binop_Projection_Add : detail::LayerBase {
  Binop_Projection_Add(View<real> const& w, View<real> const& b, bool trainable = true)
      : LayerBase(PONNI_B200_BINOP_PROJECTION_ADD, (int)w.extent(1), (int)w.extent(1)) {
    d.save_index = ISAVE;
    d.aux = (int)w.extent(0);
    params = detail::flat(w);
    auto bb = detail::flat(b);
    params.insert(params.end(), bb.begin(), bb.end());
    if (trainable) d.flags |= PONNI_B200_FLAG_TRAINABLE;
  }
};

// ---- Inference (src/ponni_Inference.h) ----
template <class real>
class Inference {
 public:
  using real1d = View<real>;
  using real2d = View<real>;

  template <class... Layers>
  explicit Inference(int device, Layers const&... layers) {
    std::vector<detail::LayerBase> ls{static_cast<detail::LayerBase const&>(layers)...};
    std::vector<ponni_b200_layer_desc> descs;
    std::vector<std::vector<real>> store(ls.size());
    for (size_t i = 0; i < ls.size(); ++i) {
      ponni_b200_layer_desc d = ls[i].d;
      store[i].resize(ls[i].params.size());
      for (size_t k = 0; k < store[i].size(); ++k) store[i][k] = real((float)ls[i].params[k]);
      if constexpr (std::is_same_v<real, double>)
        for (size_t k = 0; k < store[i].size(); ++k) store[i][k] = ls[i].params[k];
      d.params = store[i].empty() ? nullptr : store[i].data();
      descs.push_back(d);
      num_inputs_ = i == 0 ? d.num_inputs : num_inputs_;
      num_outputs_ = d.num_outputs;
    }
    ponni_b200_model* m = nullptr;
    ponni_b200_status s = ponni_b200_model_create(descs.data(), (int)descs.size(), dtype_of<real>::value, device, &m);
    if (s != PONNI_B200_OK) throw Error(s, ponni_b200_create_error());
    model_.reset(m);
  }

  void validate() const { check(ponni_b200_model_validate(model_.get())); }
  int get_num_inputs() const { return num_inputs_; }
  int get_num_outputs() const { return num_outputs_; }

  // Host batches: copies in, runs, copies out (synchronous).
  real2d forward_batch_parallel(real2d const& input) {
    real2d out("output", (size_t)num_outputs_, input.extent(1));
    forward_batch_parallel(input, out);
    return out;
  }
  void forward_batch_parallel(real2d const& input, real2d& output) {
    if ((int)input.extent(0) != num_inputs_)
      throw Error(PONNI_B200_ERR_VALIDATION, "Error: Provided # inputs differs from model's # inputs");
    if ((int)output.extent(0) != num_outputs_ || output.extent(1) != input.extent(1))
      throw Error(PONNI_B200_ERR_VALIDATION, "Error: Provided output dimensions do not match the model and input batch");
    check(ponni_b200_forward_host(model_.get(), input.data(), (int64_t)input.extent(1), output.data(),
                                  (int64_t)output.extent(1), (int64_t)input.extent(1)));
  }
  // Device batches (LayoutRight, row strides in elements); asynchronous on
  // `stream` (NULL: the model's stream), like the reference.
  void forward_batch_parallel(real const* d_in, int64_t in_ld, real* d_out, int64_t out_ld, int64_t batch,
                              void* stream = nullptr) {
    check(ponni_b200_forward(model_.get(), d_in, in_ld, d_out, out_ld, batch, stream));
  }
  void fence() { check(ponni_b200_model_synchronize(model_.get())); }

  void reallocate_internal_state(int batch) { check(ponni_b200_reallocate_internal_state(model_.get(), batch)); }
  int internal_state_capacity() const { return (int)ponni_b200_internal_state_capacity(model_.get()); }
  int get_planned_temporary_size(int which) const { return ponni_b200_planned_temporary_size(model_.get(), which); }

  int get_num_trainable_parameters() const { return (int)ponni_b200_num_trainable_parameters(model_.get()); }
  void set_trainable_parameters(real1d const& in) {
    check(ponni_b200_set_trainable_parameters(model_.get(), in.data(), (int64_t)in.size()));
  }
  real1d get_trainable_parameters() const {
    real1d out("params_glob", (size_t)get_num_trainable_parameters());
    check(ponni_b200_get_trainable_parameters(model_.get(), out.data(), (int64_t)out.size()));
    return out;
  }
  // Parameters in device memory (tuple order), written into the planned
  // model's device images on `stream` without a re-plan (generated
  // set_parameters / get_parameters, emitter.py:1787-1866).
  template <class S>
  void set_trainable_parameters_device(const S* d_src, int64_t count, void* stream = nullptr) {
    check(ponni_b200_set_trainable_parameters_device(model_.get(), d_src, dtype_of<S>::value, count, stream));
  }
  template <class S>
  void get_trainable_parameters_device(S* d_dst, int64_t count, void* stream = nullptr) const {
    check(ponni_b200_get_trainable_parameters_device(model_.get(), d_dst, dtype_of<S>::value, count, stream));
  }
  // Device checks (emitter.py:1868-1895).
  bool parameters_synchronized() const {
    int64_t mism = 0;
    check(ponni_b200_check_parameters(model_.get(), &mism, nullptr));
    return mism == 0;
  }
  bool parameters_are_finite() const {
    int64_t bad = 0;
    check(ponni_b200_check_parameters(model_.get(), nullptr, &bad));
    return bad == 0;
  }
  std::string weight_schema_fingerprint() const {
    char buf[64];
    check(ponni_b200_weight_schema_fingerprint(model_.get(), buf, sizeof buf));
    return buf;
  }
  bool save_weights(std::string const& path, std::string* error = nullptr) const {
    return file_op(ponni_b200_model_save_weights(model_.get(), path.c_str()), error);
  }
  bool load_weights(std::string const& path, std::string* error = nullptr) {
    return file_op(ponni_b200_model_load_weights(model_.get(), path.c_str()), error);
  }
  void print() const {
    std::vector<char> buf(1 << 16);
    check(ponni_b200_model_summary(model_.get(), buf.data(), buf.size()));
    std::cout << buf.data();
  }
  ponni_b200_model* handle() const { return model_.get(); }

 private:
  struct Deleter {
    void operator()(ponni_b200_model* m) const { ponni_b200_model_destroy(m); }
  };
  std::unique_ptr<ponni_b200_model, Deleter> model_;
  int num_inputs_ = 0, num_outputs_ = 0;

  void check(ponni_b200_status s) const {
    if (s != PONNI_B200_OK) throw Error(s, ponni_b200_last_error(model_.get()));
  }
  bool file_op(ponni_b200_status s, std::string* error) const {
    if (s == PONNI_B200_OK) return true;
    if (error) *error = ponni_b200_last_error(model_.get());
    return false;
  }
};

// ---- factories (src/ponni_create_model.h) ----
template <class... Layers> inline auto create_inference_model(Layers const&... layers) {
  return Inference<float>(0, layers...);
}
template <class... Layers> inline auto create_inference_model_single_precision(Layers const&... layers) {
  return Inference<float>(0, layers...);
}
template <class... Layers> inline auto create_inference_model_double_precision(Layers const&... layers) {
  return Inference<double>(0, layers...);
}
template <class... Layers> inline auto create_inference_model_half_precision(Layers const&... layers) {
  return Inference<half_t>(0, layers...);
}
template <class... Layers> inline auto create_inference_model_bhalf_precision(Layers const&... layers) {
  return Inference<bhalf_t>(0, layers...);
}

}  // namespace ponni
