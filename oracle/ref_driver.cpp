// CPU reference (test infrastructure): the reference's own template
// inference code -- its unmodified headers, src/ponni.h and everything it
// includes -- compiled against the from-scratch host Kokkos shim in
// oracle/kokkos_shim/ (OpenMP backend semantics).  Built by oracle/Makefile
// into oracle/_ref/libponni_ref.so only where the reference checkout exists;
// the tests and bench.py's reference arm use it when it is present.
//
// The reference's models are compile-time layer tuples, so each network
// structure the tests and benchmarks use is instantiated here once per
// precision (`real` = float, double, half_t, bhalf_t):
//   "mlp_relu"  [Matvec Bias ReLU]* Matvec Bias        (cfg1, cfg2, cfg3)
//   "resmlp"    Matvec Bias, 4 x [Save_State<0> LayerNorm Matvec Bias GELU
//               Matvec Bias Binop_Add<0>], Matvec Bias  (cfg4)
//   "mlp_silu"  [Matvec Bias SiLU]* Matvec Bias         (cfg5)
//   "ones"      Matvec Bias LeakyReLU(0.1)               (core unit KAT)
//   "all_kinds" every layer kind in one tuple (the all-layer-kinds GPU test:
//               activations with non-default scalars, LayerNorm, MinMaxNorm,
//               Softmax, LogSoftmax, three saved states, Binop_Add,
//               Binop_Concatenate, Binop_Projection_Add); 16-bit: without
//               ELU and SELU (see run_all_kinds)
// Widths come from `dims` (the Matvec widths in order; "mlp_*" take any
// depth up to 8 Matvecs), parameters from `params` in the reference's
// trainable order (loaded with Inference::set_trainable_parameters), inputs
// and outputs are [features, batch] in the model's storage type (fp16 /
// bf16 as raw 16-bit patterns).  The forward is the reference's
// Inference::forward_batch_parallel (src/ponni_Inference.h:339-389).
#include <omp.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "ponni.h"

static_assert(sizeof(Kokkos::Experimental::half_t) == 2 && sizeof(Kokkos::Experimental::bhalf_t) == 2,
              "16-bit types hold exactly their bits");

namespace {

using Half = Kokkos::Experimental::half_t;
using BHalf = Kokkos::Experimental::bhalf_t;

template <class real> using View1 = Kokkos::View<real*, Kokkos::LayoutRight, Kokkos::HostSpace>;
template <class real> using View2 = Kokkos::View<real**, Kokkos::LayoutRight, Kokkos::HostSpace>;

template <class real> real load(const void* p, int64_t i) {
  if constexpr (std::is_same_v<real, Half> || std::is_same_v<real, BHalf>) {
    return real::from_bits(static_cast<const uint16_t*>(p)[i]);
  } else {
    return static_cast<const real*>(p)[i];
  }
}
template <class real> void store(void* p, int64_t i, real v) {
  if constexpr (std::is_same_v<real, Half> || std::is_same_v<real, BHalf>) {
    static_cast<uint16_t*>(p)[i] = v.bits;
  } else {
    static_cast<real*>(p)[i] = v;
  }
}

template <class real, class Model>
int run(Model& model, const double* params, int64_t nparams, const void* in, int64_t in_ld, void* out,
        int64_t out_ld, int64_t batch) {
  const int need = model.get_num_trainable_parameters();
  if (nparams != need) return 3;
  View1<real> p("ref_parameters", need);
  for (int i = 0; i < need; ++i) p(i) = static_cast<real>(params[i]);
  model.set_trainable_parameters(p);
  const int nin = model.template get_num_inputs(), nout = model.template get_num_outputs();
  if (in_ld == batch && out_ld == batch) {
    // Unmanaged Views over the caller's arrays (the 16-bit types have the
    // memory layout of their bits): no copies around the forward.
    using U2 = Kokkos::View<real**, Kokkos::LayoutRight, Kokkos::HostSpace, Kokkos::MemoryTraits<Kokkos::Unmanaged>>;
    U2 x(reinterpret_cast<real*>(const_cast<void*>(in)), nin, batch);
    U2 y(reinterpret_cast<real*>(out), nout, batch);
    model.forward_batch_parallel(x, y);
    return 0;
  }
  View2<real> x("ref_input", nin, batch);
  for (int f = 0; f < nin; ++f)
    for (int64_t c = 0; c < batch; ++c) x(f, c) = load<real>(in, f * in_ld + c);
  auto y = model.forward_batch_parallel(x);
  for (size_t f = 0; f < y.extent(0); ++f)
    for (int64_t c = 0; c < batch; ++c) store<real>(out, (int64_t)f * out_ld + c, y(f, c));
  return 0;
}

template <class real> View2<real> zeros2(int a, int b) { return View2<real>("ref_w", a, b); }
template <class real> View1<real> zeros1(int a) { return View1<real>("ref_b", a); }

// [Matvec Bias Act]^(n-1) Matvec Bias with n Matvecs.
template <class real, template <class, int, class> class Act, size_t... I>
auto mlp_tuple(const int* d, std::index_sequence<I...>) {
  return std::tuple_cat(std::make_tuple(ponni::Matvec<real>(zeros2<real>(d[I], d[I + 1])),
                                        ponni::Bias<real>(zeros1<real>(d[I + 1])), Act<real, 1, Kokkos::HostSpace>(d[I + 1]))...);
}

template <class real, template <class, int, class> class Act, size_t N>
int run_mlp(const int* d, const double* params, int64_t np, const void* in, int64_t in_ld, void* out, int64_t out_ld,
            int64_t batch) {
  auto hidden = mlp_tuple<real, Act>(d, std::make_index_sequence<N - 1>());
  auto tail = std::make_tuple(ponni::Matvec<real>(zeros2<real>(d[N - 1], d[N])), ponni::Bias<real>(zeros1<real>(d[N])));
  auto model = std::apply(
      [](auto const&... layers) { return ponni::detail::create_model<real>(Kokkos::OpenMP(), Kokkos::HostSpace(), layers...); },
      std::tuple_cat(hidden, tail));
  return run<real>(model, params, np, in, in_ld, out, out_ld, batch);
}

template <class real, template <class, int, class> class Act>
int dispatch_mlp(int n, const int* d, const double* params, int64_t np, const void* in, int64_t in_ld, void* out,
                 int64_t out_ld, int64_t batch) {
  switch (n) {
    case 2: return run_mlp<real, Act, 2>(d, params, np, in, in_ld, out, out_ld, batch);
    case 3: return run_mlp<real, Act, 3>(d, params, np, in, in_ld, out, out_ld, batch);
    case 4: return run_mlp<real, Act, 4>(d, params, np, in, in_ld, out, out_ld, batch);
    case 5: return run_mlp<real, Act, 5>(d, params, np, in, in_ld, out, out_ld, batch);
    case 6: return run_mlp<real, Act, 6>(d, params, np, in, in_ld, out, out_ld, batch);
    case 7: return run_mlp<real, Act, 7>(d, params, np, in, in_ld, out, out_ld, batch);
    case 8: return run_mlp<real, Act, 8>(d, params, np, in, in_ld, out, out_ld, batch);
  }
  return 2;
}

template <class real> auto res_block(int w) {
  return std::make_tuple(ponni::Save_State<0, real>(w), ponni::LayerNorm<real>(w),
                         ponni::Matvec<real>(zeros2<real>(w, w)), ponni::Bias<real>(zeros1<real>(w)),
                         ponni::Gelu<real>(w), ponni::Matvec<real>(zeros2<real>(w, w)),
                         ponni::Bias<real>(zeros1<real>(w)), ponni::Binop_Add<0, real>(w));
}

template <class real>
int run_resmlp(const int* d, const double* params, int64_t np, const void* in, int64_t in_ld, void* out,
               int64_t out_ld, int64_t batch) {
  const int w = d[1];
  auto layers = std::tuple_cat(
      std::make_tuple(ponni::Matvec<real>(zeros2<real>(d[0], w)), ponni::Bias<real>(zeros1<real>(w))),
      res_block<real>(w), res_block<real>(w), res_block<real>(w), res_block<real>(w),
      std::make_tuple(ponni::Matvec<real>(zeros2<real>(w, d[2])), ponni::Bias<real>(zeros1<real>(d[2]))));
  auto model = std::apply(
      [](auto const&... l) { return ponni::detail::create_model<real>(Kokkos::OpenMP(), Kokkos::HostSpace(), l...); },
      layers);
  return run<real>(model, params, np, in, in_ld, out, out_ld, batch);
}

template <class real>
int run_ones(const int* d, const double* params, int64_t np, const void* in, int64_t in_ld, void* out,
             int64_t out_ld, int64_t batch) {
  auto model = ponni::detail::create_model<real>(
      Kokkos::OpenMP(), Kokkos::HostSpace(), ponni::Matvec<real>(zeros2<real>(d[0], d[1])),
      ponni::Bias<real>(zeros1<real>(d[1])), ponni::LeakyRelu<real>(d[1], static_cast<real>(0.1)));
  return run<real>(model, params, np, in, in_ld, out, out_ld, batch);
}

// ELU and SELU return `cond ? x : alpha * (std::exp(x) - 1)`, a conditional
// between a `real` and a float; for 16-bit `real` (implicit conversions both
// ways) that conditional does not compile, so the 16-bit instantiation leaves
// the two layers out ("all_kinds" without them).
template <class real>
int run_all_kinds(const int* d, const double* params, int64_t np, const void* in, int64_t in_ld, void* out,
                  int64_t out_ld, int64_t batch) {
  const int n = d[1], n2 = 2 * d[1];
  auto head = [&] {
    if constexpr (std::is_floating_point_v<real>)
      return std::make_tuple(ponni::Matvec<real>(zeros2<real>(d[0], n)), ponni::Bias<real>(zeros1<real>(n)),
                             ponni::Elu<real>(n, static_cast<real>(0.7)), ponni::Save_State<0, real>(n),
                             ponni::Selu<real>(n));
    else
      return std::make_tuple(ponni::Matvec<real>(zeros2<real>(d[0], n)), ponni::Bias<real>(zeros1<real>(n)),
                             ponni::Save_State<0, real>(n));
  }();
  auto tail = std::make_tuple(
      ponni::Softplus<real>(n, static_cast<real>(1.5)), ponni::Matvec<real>(zeros2<real>(n, n)),
      ponni::Gelu<real>(n), ponni::Gelu<real>(n, true), ponni::Mish<real>(n),
      ponni::LayerNorm<real>(zeros1<real>(n), zeros1<real>(n)), ponni::HardSigmoid<real>(n), ponni::HardSwish<real>(n),
      ponni::Binop_Add<0, real>(n), ponni::Save_State<1, real>(n), ponni::Sigmoid<real>(n), ponni::Tanh<real>(n),
      ponni::Silu<real>(n), ponni::MinMaxNorm<real>(n, static_cast<real>(-1.0), static_cast<real>(2.0)),
      ponni::Binop_Concatenate<1, real>(n, n2, true), ponni::Relu<real>(n2),
      ponni::LeakyRelu<real>(n2, static_cast<real>(0.05)), ponni::Save_State<2, real>(n2), ponni::Softmax<real>(n2),
      ponni::Binop_Projection_Add<2, real>(zeros2<real>(n2, n2), zeros1<real>(n2), true), ponni::LogSoftmax<real>(n2),
      ponni::Matvec<real>(zeros2<real>(n2, d[2])), ponni::Bias<real>(zeros1<real>(d[2])));
  auto model = std::apply(
      [](auto const&... l) { return ponni::detail::create_model<real>(Kokkos::OpenMP(), Kokkos::HostSpace(), l...); },
      std::tuple_cat(head, tail));
  return run<real>(model, params, np, in, in_ld, out, out_ld, batch);
}

template <class real>
int run_net(const std::string& net, int n_dims, const int* dims, const double* params, int64_t np, const void* in,
            int64_t in_ld, void* out, int64_t out_ld, int64_t batch) {
  if (net == "mlp_relu") return dispatch_mlp<real, ponni::Relu>(n_dims - 1, dims, params, np, in, in_ld, out, out_ld, batch);
  if (net == "mlp_silu") return dispatch_mlp<real, ponni::Silu>(n_dims - 1, dims, params, np, in, in_ld, out, out_ld, batch);
  if (net == "resmlp" && n_dims == 3) return run_resmlp<real>(dims, params, np, in, in_ld, out, out_ld, batch);
  if (net == "ones" && n_dims == 2) return run_ones<real>(dims, params, np, in, in_ld, out, out_ld, batch);
  if (net == "all_kinds" && n_dims == 3) return run_all_kinds<real>(dims, params, np, in, in_ld, out, out_ld, batch);
  return 1;
}

}  // namespace

extern "C" {

// dtype: 0 fp32, 1 fp64, 2 fp16, 3 bf16 (ponni_b200_dtype).  Returns 0 on
// success, 1 unknown network, 2 unsupported depth, 3 parameter count
// mismatch.  nthreads <= 0 keeps the OpenMP default.
int ponni_ref_forward(const char* net, int dtype, int n_dims, const int* dims, const double* params, int64_t nparams,
                      const void* in, int64_t in_ld, void* out, int64_t out_ld, int64_t batch, int nthreads) {
  if (nthreads > 0) omp_set_num_threads(nthreads);
  const std::string n(net);
  switch (dtype) {
    case 0: return run_net<float>(n, n_dims, dims, params, nparams, in, in_ld, out, out_ld, batch);
    case 1: return run_net<double>(n, n_dims, dims, params, nparams, in, in_ld, out, out_ld, batch);
    case 2: return run_net<Half>(n, n_dims, dims, params, nparams, in, in_ld, out, out_ld, batch);
    case 3: return run_net<BHalf>(n, n_dims, dims, params, nparams, in, in_ld, out, out_ld, batch);
  }
  return 4;
}

}  // extern "C"
