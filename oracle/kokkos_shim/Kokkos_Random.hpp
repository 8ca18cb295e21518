// Host random generator with the Kokkos::Random_XorShift64 interface used by
// the reference's initializers (written from scratch for the host Kokkos
// shim; its stream is not Kokkos' and the tests never use it: weights are
// always passed explicitly).
#pragma once
#include <cmath>
#include <cstdint>

#include "Kokkos_Core.hpp"

namespace Kokkos {

template <class ExecutionSpace> class Random_XorShift64 {
  std::uint64_t state_;

 public:
  explicit Random_XorShift64(std::uint64_t state = 1, int = 0) : state_(state ? state : 0x9e3779b97f4a7c15ull) {}
  std::uint64_t urand64() {
    state_ ^= state_ >> 12;
    state_ ^= state_ << 25;
    state_ ^= state_ >> 27;
    return state_ * 0x2545f4914f6cdd1dull;
  }
  std::uint32_t urand() { return (std::uint32_t)(urand64() >> 32); }
  double drand() { return (double)(urand64() >> 11) * (1.0 / 9007199254740992.0); }
  double drand(double r) { return r * drand(); }
  double drand(double a, double b) { return a + (b - a) * drand(); }
  float frand() { return (float)drand(); }
  float frand(float a, float b) { return a + (b - a) * frand(); }
  double normal() {
    const double u1 = (drand() * 0.999999999) + 1e-12, u2 = drand();
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
  }
  double normal(double mean, double stdev) { return mean + stdev * normal(); }
};

}  // namespace Kokkos
