// C++ drop-in API test (include/ponni_b200.hpp), following the reference's
// unit/core/test_core_unit.cpp:200-377 known-answer tests.
//   ./test_template_api host   -- construction, validation, fingerprint, .ponni round trip
//   ./test_template_api gpu    -- forward passes on the GPU
#include <cmath>
#include <cstdio>
#include <string>

#include "ponni_b200.hpp"

static int failures = 0;
#define REQUIRE(c, msg)                                   \
  do {                                                    \
    if (!(c)) {                                           \
      std::fprintf(stderr, "FAILED: %s (%s)\n", msg, #c); \
      ++failures;                                         \
    }                                                     \
  } while (0)

static bool near(float a, float b, float tol = 1e-5f) { return std::fabs(a - b) <= tol; }

using real2d = ponni::View<float>;

static auto ones_model() {
  real2d w("w", 2, 2);
  ponni::View<float> b("b", 2);
  ponni::deep_copy(w, 1.0f);
  ponni::deep_copy(b, 1.0f);
  return ponni::create_inference_model(ponni::Matvec<float>(w), ponni::Bias<float>(b), ponni::LeakyRelu<float>(2, 0.1));
}

static void host_tests() {
  auto model = ones_model();
  model.validate();
  REQUIRE(model.get_num_trainable_parameters() == 6, "trainable count");
  REQUIRE(model.weight_schema_fingerprint().rfind("fnv1a64:", 0) == 0, "fingerprint format");
  std::string err;
  REQUIRE(model.save_weights("cpp_template_weights.ponni", &err), "save");
  ponni::View<float> zeros("z", 6);
  model.set_trainable_parameters(zeros);
  REQUIRE(model.get_trainable_parameters()(0) == 0.0f, "set params");
  REQUIRE(model.load_weights("cpp_template_weights.ponni", &err), "load");
  REQUIRE(model.get_trainable_parameters()(5) == 1.0f, "params restored");
  std::remove("cpp_template_weights.ponni");
  // four-block planning: tmp1 7, tmp2 3 (test_core_unit.cpp:320-323)
  real2d w1("w1", 2, 5), w2("w2", 5, 3), w3("w3", 3, 7), w4("w4", 7, 2);
  ponni::View<float> b1("b1", 5), b2("b2", 3), b3("b3", 7), b4("b4", 2);
  auto fm = ponni::create_inference_model(ponni::Matvec<float>(w1), ponni::Bias<float>(b1), ponni::Relu<float>(5),
                                          ponni::Tanh<float>(5), ponni::Matvec<float>(w2), ponni::Bias<float>(b2),
                                          ponni::Sigmoid<float>(3), ponni::Matvec<float>(w3), ponni::Bias<float>(b3),
                                          ponni::LeakyRelu<float>(7, 0.2), ponni::Matvec<float>(w4),
                                          ponni::Bias<float>(b4), ponni::HardSwish<float>(2));
  REQUIRE(fm.get_planned_temporary_size(0) == 7 && fm.get_planned_temporary_size(1) == 3, "planned sizes");
  // validation failure mirrors Kokkos::abort
  real2d wbad("wb", 2, 3);
  ponni::View<float> bbad("bb", 4);
  auto bad = ponni::create_inference_model(ponni::Matvec<float>(wbad), ponni::Bias<float>(bbad));
  bool threw = false;
  try {
    bad.validate();
  } catch (ponni::Error const& e) {
    threw = e.status == PONNI_B200_ERR_VALIDATION;
  }
  REQUIRE(threw, "validate throws on mismatch");
  auto half_model = ponni::create_inference_model_half_precision(ponni::Relu<ponni::half_t>(3));
  REQUIRE(half_model.get_num_inputs() == 3, "half factory");
}

static void gpu_tests() {
  auto model = ones_model();
  real2d in("in", 2, 1);
  in(0, 0) = 1.0f;
  in(1, 0) = 2.0f;
  auto out = model.forward_batch_parallel(in);
  REQUIRE(near(out(0, 0), 4.0f) && near(out(1, 0), 4.0f), "ones network -> 4,4");
  REQUIRE(model.internal_state_capacity() == 1, "capacity 1");
  real2d big("big", 2, 4);
  ponni::deep_copy(big, 1.0f);
  model.forward_batch_parallel(big);
  REQUIRE(model.internal_state_capacity() == 4, "capacity grows");
  model.reallocate_internal_state(2);
  REQUIRE(model.internal_state_capacity() == 2, "capacity shrinks");
  // README 2->3->1 -> 0.7
  real2d w1("w1", 2, 3), w2("w2", 3, 1);
  ponni::View<float> b1("b1", 3), b2("b2", 1);
  ponni::deep_copy(w1, 0.25f);
  ponni::deep_copy(b1, 0.10f);
  ponni::deep_copy(w2, 0.50f);
  ponni::deep_copy(b2, -0.20f);
  auto readme = ponni::create_inference_model(ponni::Matvec<float>(w1), ponni::Bias<float>(b1), ponni::Relu<float>(3),
                                              ponni::Matvec<float>(w2), ponni::Bias<float>(b2));
  readme.validate();
  real2d x("x", 2, 100000);
  ponni::deep_copy(x, 1.0f);
  auto y = readme.forward_batch_parallel(x);
  REQUIRE(near(y(0, 0), 0.7f, 1e-6f) && near(y(0, 99999), 0.7f, 1e-6f), "README -> 0.7");
  // parameter update of the planned model (device scatter, no re-plan)
  auto p = readme.get_trainable_parameters();
  REQUIRE(p.size() == 2 * 3 + 3 + 3 + 1, "trainable count");
  p(p.size() - 1) = 0.8f;  // b2: -0.2 -> 0.8
  readme.set_trainable_parameters(p);
  y = readme.forward_batch_parallel(x);
  REQUIRE(near(y(0, 0), 1.7f, 1e-6f) && near(y(0, 99999), 1.7f, 1e-6f), "updated bias -> 1.7");
  REQUIRE(readme.parameters_synchronized() && readme.parameters_are_finite(), "device images in step");
  // double and half models
  ponni::View<double> wd("wd", 2, 2);
  ponni::deep_copy(wd, 1.0);
  auto dm = ponni::create_inference_model_double_precision(ponni::Matvec<double>(wd));
  ponni::View<double> xd("xd", 2, 1);
  xd(0, 0) = 1.0;
  xd(1, 0) = 2.0;
  auto yd = dm.forward_batch_parallel(xd);
  REQUIRE(yd(0, 0) == 3.0 && yd(1, 0) == 3.0, "double model");
  ponni::View<ponni::half_t> wh("wh", 3, 1);
  ponni::deep_copy(wh, ponni::half_t(1.0f));
  auto hm = ponni::create_inference_model_half_precision(ponni::Matvec<ponni::half_t>(wh));
  ponni::View<ponni::half_t> xh("xh", 3, 1);
  xh(0, 0) = 2048.0f;
  xh(1, 0) = 1.0f;
  xh(2, 0) = 1.0f;
  auto yh = hm.forward_batch_parallel(xh);
  REQUIRE((float)yh(0, 0) == 2048.0f, "half model accumulates in half");
}

int main(int argc, char** argv) {
  std::string mode = argc > 1 ? argv[1] : "host";
  try {
    if (mode == "host") host_tests();
    else gpu_tests();
  } catch (std::exception const& e) {
    std::fprintf(stderr, "exception: %s\n", e.what());
    return 2;
  }
  if (failures) return 1;
  std::printf("ok %s\n", mode.c_str());
  return 0;
}
