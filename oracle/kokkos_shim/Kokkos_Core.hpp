// A minimal host-only Kokkos API, written from scratch for one purpose: to
// compile the reference's unmodified headers (src/ponni.h and what it
// includes) as a CPU oracle and CPU baseline (test infrastructure, never the
// product).  It provides only the names those headers use, with the
// semantics of Kokkos' OpenMP backend on a host:
//   * one execution space (OpenMP) and one memory space (HostSpace);
//   * View<T*...> of rank 1-4, LayoutRight, reference-counted storage,
//     unmanaged views over caller memory, label, extents;
//   * realloc / view_alloc / WithoutInitializing, deep_copy, subview with
//     index pairs, create_mirror_view[_and_copy];
//   * parallel_for / parallel_reduce over RangePolicy (OpenMP static
//     schedule), Sum reducer, fence, abort;
//   * the math functions PONNI calls, bit_cast;
//   * Experimental::half_t and bhalf_t as IEEE binary16 / bfloat16 storage
//     whose arithmetic runs in float and rounds every result to the type
//     (round to nearest even): the behaviour of Kokkos' half types on hosts
//     without native 16-bit arithmetic.
// No Kokkos source is used; Kokkos is not present in this checkout.
#pragma once

#include <omp.h>

#include <algorithm>
#include <array>
#include <bit>
#include <cmath>
#include <functional>
#include <iostream>
#include <tuple>
#include <vector>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <memory>
#include <string>
#include <type_traits>
#include <utility>

#define KOKKOS_INLINE_FUNCTION inline
#define KOKKOS_FORCEINLINE_FUNCTION inline
#define KOKKOS_FUNCTION
#define KOKKOS_LAMBDA [=]
#define KOKKOS_CLASS_LAMBDA [=, *this]
#define KOKKOS_ENABLE_OPENMP 1
#define KOKKOS_SHIM_STRIP(...) __VA_ARGS__
#define KOKKOS_IF_ON_HOST(CODE) {KOKKOS_SHIM_STRIP CODE}
#define KOKKOS_IF_ON_DEVICE(CODE) \
  {}

namespace Kokkos {

// ------------------------------------------------------------------ spaces --
struct HostSpace;
struct OpenMP {
  using execution_space = OpenMP;
  using memory_space = HostSpace;
  using size_type = std::size_t;
  void fence(const std::string& = std::string()) const {}
  static int concurrency() { return omp_get_max_threads(); }
  static const char* name() { return "OpenMP"; }
};
struct HostSpace {
  using memory_space = HostSpace;
  using execution_space = OpenMP;
  using size_type = std::size_t;
  static const char* name() { return "Host"; }
};
using DefaultExecutionSpace = OpenMP;
using DefaultHostExecutionSpace = OpenMP;
using Serial = OpenMP;

template <class T> struct is_execution_space : std::false_type {};
template <> struct is_execution_space<OpenMP> : std::true_type {};
template <class T> inline constexpr bool is_execution_space_v = is_execution_space<std::remove_cv_t<T>>::value;
template <class T> struct is_memory_space : std::false_type {};
template <> struct is_memory_space<HostSpace> : std::true_type {};
template <class T> inline constexpr bool is_memory_space_v = is_memory_space<std::remove_cv_t<T>>::value;
template <class A, class B> struct SpaceAccessibility {
  static constexpr bool accessible = true;
  static constexpr bool assignable = true;
};

inline void fence(const std::string& = std::string()) {}

[[noreturn]] inline void abort(const char* msg) {
  std::fprintf(stderr, "%s\n", msg);
  std::fflush(stderr);
  std::abort();
}

using std::printf;

template <class To, class From> inline To bit_cast(const From& f) { return std::bit_cast<To>(f); }

// ---------------------------------------------------------------- layouts --
struct LayoutRight {};
struct LayoutLeft {};
struct LayoutStride {};

enum MemoryTraitsFlags : unsigned { Unmanaged = 0x01, RandomAccess = 0x02, Atomic = 0x04, Restrict = 0x08 };
template <unsigned Flags> struct MemoryTraits {
  static constexpr unsigned value = Flags;
  static constexpr bool is_unmanaged = (Flags & Unmanaged) != 0;
};

// ------------------------------------------------------------- half types --
namespace Experimental {
namespace shim {
// float -> IEEE binary16 bits, round to nearest even (constexpr: PONNI
// declares constexpr constants of its `real` type).
constexpr std::uint16_t float_to_half_bits(float f) {
  const std::uint32_t x = std::bit_cast<std::uint32_t>(f);
  const std::uint32_t sign = (x >> 16) & 0x8000u;
  const std::uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (std::uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (std::uint16_t)(sign | 0x7c00u);  // rounds to infinity
  if (ax >= 0x38800000u) {                                        // normal in binary16
    std::uint32_t r = ax - 0x38000000u;                            // rebias 127 -> 15
    r += 0xfffu + ((r >> 13) & 1u);
    return (std::uint16_t)(sign | (r >> 13));
  }
  if (ax <= 0x33000000u) return (std::uint16_t)sign;  // at most 2^-25: rounds to zero (ties to even)
  // subnormal in binary16: units of 2^-24
  const std::uint32_t e = ax >> 23;
  const std::uint32_t m = (ax & 0x7fffffu) | 0x800000u;
  const std::uint32_t sh = 126u - e;
  std::uint32_t q = m >> sh;
  const std::uint32_t rem = m & ((1u << sh) - 1u), halfway = 1u << (sh - 1u);
  if (rem > halfway || (rem == halfway && (q & 1u))) ++q;
  return (std::uint16_t)(sign | q);
}
constexpr float half_bits_to_float(std::uint16_t h) {
  const std::uint32_t sign = (std::uint32_t)(h & 0x8000u) << 16;
  const std::uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  if (e == 0) {
    const float v = (float)m * (1.0f / 16777216.0f);
    return sign ? -v : v;
  }
  if (e == 31) return std::bit_cast<float>(sign | 0x7f800000u | (m << 13));
  return std::bit_cast<float>(sign | ((e + 112u) << 23) | (m << 13));
}
constexpr std::uint16_t float_to_bhalf_bits(float f) {
  const std::uint32_t x = std::bit_cast<std::uint32_t>(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (std::uint16_t)((x >> 16) | 0x40u);  // quiet NaN
  return (std::uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
}
constexpr float bhalf_bits_to_float(std::uint16_t h) { return std::bit_cast<float>((std::uint32_t)h << 16); }

// A 16-bit floating type in the manner of Kokkos' host half types:
// constructible from arithmetic values (rounded), converted implicitly to
// float (explicitly to double); operations between two values of the type
// run in float and round the result to the type; mixed operations with float
// or double are carried out in that type (compound assignments round the
// result once).
template <std::uint16_t (*ToBits)(float), float (*FromBits)(std::uint16_t)>
struct Half16 {
  std::uint16_t bits;  // (uninitialised by default: arrays allocated without initialising stay untouched)
  Half16() = default;
  template <class T, class = std::enable_if_t<std::is_arithmetic_v<T>>>
  constexpr Half16(T v) : bits(ToBits((float)v)) {}
  static constexpr Half16 from_bits(std::uint16_t b) {
    Half16 h{};
    h.bits = b;
    return h;
  }
  constexpr operator float() const { return FromBits(bits); }
  constexpr explicit operator double() const { return (double)FromBits(bits); }
  constexpr Half16& operator+=(Half16 o) { return *this = Half16((float)*this + (float)o); }
  constexpr Half16& operator-=(Half16 o) { return *this = Half16((float)*this - (float)o); }
  constexpr Half16& operator*=(Half16 o) { return *this = Half16((float)*this * (float)o); }
  constexpr Half16& operator/=(Half16 o) { return *this = Half16((float)*this / (float)o); }
  // compound operations with a float / double right-hand side run in that type
  // and round once
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>
  constexpr Half16& operator+=(T o) { return *this = Half16((T)(float)*this + o); }
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>
  constexpr Half16& operator-=(T o) { return *this = Half16((T)(float)*this - o); }
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>
  constexpr Half16& operator*=(T o) { return *this = Half16((T)(float)*this * o); }
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>
  constexpr Half16& operator/=(T o) { return *this = Half16((T)(float)*this / o); }
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>
  friend constexpr T& operator+=(T& a, Half16 b) { return a += (T)(float)b; }
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>
  friend constexpr T& operator-=(T& a, Half16 b) { return a -= (T)(float)b; }
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>
  friend constexpr T& operator*=(T& a, Half16 b) { return a *= (T)(float)b; }
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>
  friend constexpr T& operator/=(T& a, Half16 b) { return a /= (T)(float)b; }
  constexpr Half16 operator-() const { return from_bits((std::uint16_t)(bits ^ 0x8000u)); }
  constexpr Half16 operator+() const { return *this; }
#define KOKKOS_SHIM_HALF_BINARY(OP)                                                                    \
  friend constexpr Half16 operator OP(Half16 a, Half16 b) { return Half16((float)a OP(float) b); }     \
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>                           \
  friend constexpr T operator OP(Half16 a, T b) {                                                      \
    return (T)(float)a OP b;                                                                           \
  }                                                                                                    \
  template <class T, class = std::enable_if_t<std::is_floating_point_v<T>>>                           \
  friend constexpr T operator OP(T a, Half16 b) {                                                      \
    return a OP(T)(float) b;                                                                           \
  }                                                                                                    \
  template <class T, class = std::enable_if_t<std::is_integral_v<T>>, class = void>                   \
  friend constexpr Half16 operator OP(Half16 a, T b) {                                                 \
    return a OP Half16(b);                                                                             \
  }                                                                                                    \
  template <class T, class = std::enable_if_t<std::is_integral_v<T>>, class = void>                   \
  friend constexpr Half16 operator OP(T a, Half16 b) {                                                 \
    return Half16(a) OP b;                                                                             \
  }
  KOKKOS_SHIM_HALF_BINARY(+)
  KOKKOS_SHIM_HALF_BINARY(-)
  KOKKOS_SHIM_HALF_BINARY(*)
  KOKKOS_SHIM_HALF_BINARY(/)
#undef KOKKOS_SHIM_HALF_BINARY
#define KOKKOS_SHIM_HALF_COMPARE(OP)                                                                   \
  friend constexpr bool operator OP(Half16 a, Half16 b) { return (float)a OP(float) b; }               \
  template <class T, class = std::enable_if_t<std::is_arithmetic_v<T>>>                               \
  friend constexpr bool operator OP(Half16 a, T b) {                                                   \
    return (double)(float)a OP(double) b;                                                              \
  }                                                                                                    \
  template <class T, class = std::enable_if_t<std::is_arithmetic_v<T>>>                               \
  friend constexpr bool operator OP(T a, Half16 b) {                                                   \
    return (double)a OP(double)(float) b;                                                              \
  }
  KOKKOS_SHIM_HALF_COMPARE(<)
  KOKKOS_SHIM_HALF_COMPARE(>)
  KOKKOS_SHIM_HALF_COMPARE(<=)
  KOKKOS_SHIM_HALF_COMPARE(>=)
  KOKKOS_SHIM_HALF_COMPARE(==)
  KOKKOS_SHIM_HALF_COMPARE(!=)
#undef KOKKOS_SHIM_HALF_COMPARE
};
}  // namespace shim

using half_t = shim::Half16<shim::float_to_half_bits, shim::half_bits_to_float>;
using bhalf_t = shim::Half16<shim::float_to_bhalf_bits, shim::bhalf_bits_to_float>;

template <class T> inline constexpr T quiet_NaN_v = std::numeric_limits<T>::quiet_NaN();
template <class T> inline constexpr T infinity_v = std::numeric_limits<T>::infinity();
template <class T> inline constexpr T epsilon_v = std::numeric_limits<T>::epsilon();

inline half_t cast_to_half(float v) { return half_t(v); }
inline half_t cast_to_half(double v) { return half_t((float)v); }
template <class T> inline T cast_from_half(half_t h) { return (T)(float)h; }
inline bhalf_t cast_to_bhalf(float v) { return bhalf_t(v); }
template <class T> inline T cast_from_bhalf(bhalf_t h) { return (T)(float)h; }
}  // namespace Experimental

template <class T>
inline constexpr bool is_half_v =
    std::is_same_v<T, Experimental::half_t> || std::is_same_v<T, Experimental::bhalf_t>;

// ------------------------------------------------------------------- math --
#define KOKKOS_SHIM_UNARY(NAME)                                                          \
  inline float NAME(float x) { return std::NAME(x); }                                    \
  inline double NAME(double x) { return std::NAME(x); }                                  \
  inline Experimental::half_t NAME(Experimental::half_t x) {                             \
    return Experimental::half_t(std::NAME((float)x));                                    \
  }                                                                                      \
  inline Experimental::bhalf_t NAME(Experimental::bhalf_t x) {                           \
    return Experimental::bhalf_t(std::NAME((float)x));                                   \
  }                                                                                      \
  template <class T, class = std::enable_if_t<std::is_integral_v<T>>>                    \
  inline double NAME(T x) {                                                              \
    return std::NAME((double)x);                                                         \
  }
KOKKOS_SHIM_UNARY(exp)
KOKKOS_SHIM_UNARY(expm1)
KOKKOS_SHIM_UNARY(log)
KOKKOS_SHIM_UNARY(log1p)
KOKKOS_SHIM_UNARY(tanh)
KOKKOS_SHIM_UNARY(erf)
KOKKOS_SHIM_UNARY(sqrt)
KOKKOS_SHIM_UNARY(floor)
KOKKOS_SHIM_UNARY(ceil)
KOKKOS_SHIM_UNARY(sin)
KOKKOS_SHIM_UNARY(cos)
KOKKOS_SHIM_UNARY(tan)
KOKKOS_SHIM_UNARY(sinh)
KOKKOS_SHIM_UNARY(cosh)
KOKKOS_SHIM_UNARY(asin)
KOKKOS_SHIM_UNARY(acos)
KOKKOS_SHIM_UNARY(atan)
KOKKOS_SHIM_UNARY(asinh)
KOKKOS_SHIM_UNARY(acosh)
KOKKOS_SHIM_UNARY(atanh)
KOKKOS_SHIM_UNARY(round)
#undef KOKKOS_SHIM_UNARY
inline float abs(float x) { return std::fabs(x); }
inline double abs(double x) { return std::fabs(x); }
inline int abs(int x) { return std::abs(x); }
inline Experimental::half_t abs(Experimental::half_t x) { return Experimental::half_t(std::fabs((float)x)); }
inline Experimental::bhalf_t abs(Experimental::bhalf_t x) { return Experimental::bhalf_t(std::fabs((float)x)); }
inline float pow(float a, float b) { return std::pow(a, b); }
inline double pow(double a, double b) { return std::pow(a, b); }
template <class T> inline bool isinf(T x) { return std::isinf((double)x); }
template <class T> inline bool isnan(T x) { return std::isnan((double)x); }
template <class T> inline bool isfinite(T x) { return std::isfinite((double)x); }
template <class T> inline T max(T a, T b) { return a < b ? b : a; }
template <class T> inline T min(T a, T b) { return b < a ? b : a; }

// ------------------------------------------------------------------- views --
namespace shim {
template <class T> struct DataOf {
  using value = T;
  static constexpr int rank = 0;
};
template <class T> struct DataOf<T*> {
  using value = typename DataOf<T>::value;
  static constexpr int rank = DataOf<T>::rank + 1;
};
template <class T, int R> struct AddPointers { using type = typename AddPointers<T*, R - 1>::type; };
template <class T> struct AddPointers<T, 0> { using type = T; };

template <class... P> struct Props {
  using layout = LayoutRight;
  using space = HostSpace;
  static constexpr unsigned traits = 0;
};
template <class P0, class... P> struct Props<P0, P...> : Props<P...> {
  using layout = std::conditional_t<std::is_same_v<P0, LayoutRight> || std::is_same_v<P0, LayoutLeft> ||
                                        std::is_same_v<P0, LayoutStride>,
                                    P0, typename Props<P...>::layout>;
  using space = std::conditional_t<is_memory_space_v<P0>, P0,
                                   std::conditional_t<is_execution_space_v<P0>, HostSpace, typename Props<P...>::space>>;
};
template <unsigned F, class... P> struct Props<MemoryTraits<F>, P...> : Props<P...> {
  static constexpr unsigned traits = F;
};

struct ViewAllocProp {
  std::string label;
  bool initialize = true;
};
// One allocation and its label (shared by every view of it).
struct Record {
  std::string label;
  unsigned char* mem;
  Record(std::size_t bytes, const std::string& l) : label(l), mem(new unsigned char[bytes ? bytes : 1]) {}
  ~Record() { delete[] mem; }
  Record(const Record&) = delete;
  Record& operator=(const Record&) = delete;
};
}  // namespace shim

struct WithoutInitializing_t {};
inline constexpr WithoutInitializing_t WithoutInitializing{};
struct ALL_t {};
inline constexpr ALL_t ALL{};

namespace shim {
inline void apply_alloc_arg(ViewAllocProp& p, const std::string& s) { p.label = s; }
inline void apply_alloc_arg(ViewAllocProp& p, const char* s) { p.label = s; }
inline void apply_alloc_arg(ViewAllocProp& p, WithoutInitializing_t) { p.initialize = false; }
template <class T> inline void apply_alloc_arg(ViewAllocProp&, const T&) {}  // execution space instances
}  // namespace shim

template <class... A> inline shim::ViewAllocProp view_alloc(const A&... a) {
  shim::ViewAllocProp p;
  (shim::apply_alloc_arg(p, a), ...);
  return p;
}

template <class DataType, class... Properties> class View {
  using P = shim::Props<Properties...>;

 public:
  using data_type = DataType;
  using value_type = typename shim::DataOf<DataType>::value;
  using non_const_value_type = std::remove_const_t<value_type>;
  using const_value_type = const non_const_value_type;
  static constexpr int rank = shim::DataOf<DataType>::rank;
  static constexpr int rank_dynamic = rank;
  using non_const_data_type = typename shim::AddPointers<non_const_value_type, rank>::type;
  using const_data_type = typename shim::AddPointers<const_value_type, rank>::type;
  using array_layout = typename P::layout;
  using memory_space = typename P::space;
  using execution_space = typename memory_space::execution_space;
  using device_type = memory_space;
  using memory_traits = MemoryTraits<P::traits>;
  using size_type = std::size_t;
  using index_type = std::int64_t;
  using pointer_type = value_type*;
  using reference_type = value_type&;
  using non_const_type = View<non_const_data_type, Properties...>;
  using const_type = View<const_data_type, Properties...>;
  using HostMirror = View<non_const_data_type, LayoutRight, HostSpace>;

  static_assert(rank >= 1 && rank <= 4, "the shim's Views have rank 1 to 4");

  View() = default;

  template <class... I, class = std::enable_if_t<(std::is_integral_v<I> && ...)>>
  explicit View(const std::string& label, I... n) {
    allocate(shim::ViewAllocProp{label, true}, n...);
  }
  template <class... I, class = std::enable_if_t<(std::is_integral_v<I> && ...)>>
  explicit View(const char* label, I... n) {
    allocate(shim::ViewAllocProp{label, true}, n...);
  }
  template <class... I, class = std::enable_if_t<(std::is_integral_v<I> && ...)>>
  explicit View(const shim::ViewAllocProp& p, I... n) {
    allocate(p, n...);
  }
  // Unmanaged view over caller memory.
  template <class... I, class = std::enable_if_t<(std::is_integral_v<I> && ...)>>
  View(value_type* p, I... n) {
    set_extents(n...);
    ptr_ = p;
  }
  // Conversions between compatible views (non-const -> const, other properties).
  template <class D2, class... P2,
            class = std::enable_if_t<View<D2, P2...>::rank == rank &&
                                     std::is_convertible_v<typename View<D2, P2...>::value_type*, value_type*>>>
  View(const View<D2, P2...>& o) : rec_(o.rec_), ptr_(o.ptr_) {
    if (!omp_in_parallel()) owner_ = o.owner_;
    for (int i = 0; i < 8; ++i) ext_[i] = o.ext_[i];
  }

  std::size_t extent(int i) const { return i < rank ? ext_[i] : 1; }
  int extent_int(int i) const { return (int)extent(i); }
  std::size_t size() const {
    std::size_t s = 1;
    for (int i = 0; i < rank; ++i) s *= ext_[i];
    return s;
  }
  std::size_t span() const { return size(); }
  value_type* data() const { return ptr_; }
  std::string label() const { return rec_ ? rec_->label : std::string(); }
  bool is_allocated() const { return ptr_ != nullptr; }
  int use_count() const { return (int)owner_.use_count(); }
  std::size_t stride(int i) const {
    std::size_t s = 1;
    for (int k = rank - 1; k > i; --k) s *= ext_[k];
    return s;
  }

  template <class I0> value_type& operator()(I0 i0) const {
    static_assert(rank == 1, "rank-1 access");
    return ptr_[i0];
  }
  template <class I0, class I1> value_type& operator()(I0 i0, I1 i1) const {
    static_assert(rank == 2, "rank-2 access");
    return ptr_[(std::size_t)i0 * ext_[1] + (std::size_t)i1];
  }
  template <class I0, class I1, class I2> value_type& operator()(I0 i0, I1 i1, I2 i2) const {
    static_assert(rank == 3, "rank-3 access");
    return ptr_[((std::size_t)i0 * ext_[1] + (std::size_t)i1) * ext_[2] + (std::size_t)i2];
  }
  template <class I0, class I1, class I2, class I3> value_type& operator()(I0 i0, I1 i1, I2 i2, I3 i3) const {
    static_assert(rank == 4, "rank-4 access");
    return ptr_[(((std::size_t)i0 * ext_[1] + (std::size_t)i1) * ext_[2] + (std::size_t)i2) * ext_[3] +
                (std::size_t)i3];
  }
  template <class I0> value_type& operator[](I0 i0) const { return ptr_[i0]; }

  // shim internals (public so that views of other types can share them).
  // Like Kokkos, a copy made inside a parallel region does not take part in
  // the reference counting (no atomic traffic per sample): it points at the
  // allocation record without owning it.
  std::shared_ptr<shim::Record> owner_;
  shim::Record* rec_ = nullptr;
  value_type* ptr_ = nullptr;
  std::size_t ext_[8] = {0, 0, 0, 0, 0, 0, 0, 0};

  View(const View& o) : rec_(o.rec_), ptr_(o.ptr_) {
    if (!omp_in_parallel()) owner_ = o.owner_;
    for (int i = 0; i < 8; ++i) ext_[i] = o.ext_[i];
  }
  View& operator=(const View& o) {
    if (this != &o) {
      if (!omp_in_parallel()) owner_ = o.owner_;
      else owner_.reset();
      rec_ = o.rec_;
      ptr_ = o.ptr_;
      for (int i = 0; i < 8; ++i) ext_[i] = o.ext_[i];
    }
    return *this;
  }

 private:
  template <class... I> void set_extents(I... n) {
    static_assert(sizeof...(I) == rank, "one extent per rank");
    const std::size_t e[] = {(std::size_t)n...};
    for (int i = 0; i < rank; ++i) ext_[i] = e[i];
  }
  template <class... I> void allocate(const shim::ViewAllocProp& p, I... n) {
    set_extents(n...);
    const std::size_t s = size() ? size() : 1;
    if (p.initialize) {
      // value-initialised in parallel (first touch by the threads that use it)
      non_const_value_type* q = raw_alloc(s, p.label);
#pragma omp parallel for schedule(static)
      for (std::int64_t i = 0; i < (std::int64_t)s; ++i) q[i] = non_const_value_type();
      ptr_ = q;
    } else {
      ptr_ = raw_alloc(s, p.label);  // WithoutInitializing: no construction, no touch
    }
  }
  non_const_value_type* raw_alloc(std::size_t s, const std::string& label = std::string()) {
    static_assert(std::is_trivially_copyable_v<non_const_value_type>, "the shim's Views hold trivial types");
    owner_ = std::make_shared<shim::Record>(s * sizeof(non_const_value_type), label);
    rec_ = owner_.get();
    return reinterpret_cast<non_const_value_type*>(rec_->mem);
  }
};

template <class T> struct is_view : std::false_type {};
template <class D, class... P> struct is_view<View<D, P...>> : std::true_type {};
template <class T> inline constexpr bool is_view_v = is_view<std::remove_cv_t<T>>::value;

template <class V, class... I> inline void realloc(V& v, I... n) {
  v = V(shim::ViewAllocProp{v.label(), true}, n...);
}
template <class V, class... I> inline void realloc(const shim::ViewAllocProp& p, V& v, I... n) {
  shim::ViewAllocProp q = p;
  if (q.label.empty()) q.label = v.label();
  v = V(q, n...);
}
template <class V, class... I> inline void resize(V& v, I... n) {
  V w(shim::ViewAllocProp{v.label(), true}, n...);
  const std::size_t m = std::min(v.size(), w.size());
  for (std::size_t i = 0; i < m; ++i) w.data()[i] = v.data()[i];
  v = w;
}

template <class D1, class... P1, class D2, class... P2>
inline void deep_copy(const View<D1, P1...>& dst, const View<D2, P2...>& src) {
  if (dst.size() != src.size()) abort("Kokkos::deep_copy: extents differ");
  using T = typename View<D1, P1...>::non_const_value_type;
  for (std::size_t i = 0; i < dst.size(); ++i) dst.data()[i] = (T)src.data()[i];
}
template <class D1, class... P1, class S, class = std::enable_if_t<!is_view_v<S>>>
inline void deep_copy(const View<D1, P1...>& dst, const S& value) {
  using T = typename View<D1, P1...>::non_const_value_type;
  for (std::size_t i = 0; i < dst.size(); ++i) dst.data()[i] = (T)value;
}
template <class E, class A, class B, class = std::enable_if_t<is_execution_space_v<E>>>
inline void deep_copy(const E&, const A& dst, const B& src) {
  deep_copy(dst, src);
}

template <class V> inline typename V::HostMirror create_mirror_view(const V& v) {
  return typename V::HostMirror(v);
}
template <class V> inline typename V::HostMirror create_mirror(const V& v) {
  typename V::HostMirror m(shim::ViewAllocProp{v.label(), true}, v.extent(0));
  return m;
}
// Same (host) memory space: Kokkos returns the view itself.
template <class S, class D, class... P>
inline View<typename View<D, P...>::non_const_data_type, LayoutRight, HostSpace> create_mirror_view_and_copy(
    const S&, const View<D, P...>& v) {
  using R = View<typename View<D, P...>::non_const_data_type, LayoutRight, HostSpace>;
  R r;
  r.owner_ = v.owner_;
  r.rec_ = v.rec_;
  r.ptr_ = const_cast<typename R::value_type*>(v.data());
  for (int i = 0; i < 8; ++i) r.ext_[i] = v.ext_[i];
  return r;
}

// Contiguous sub-ranges of rank-1 views.
template <class D, class... P, class I>
inline View<D, P...> subview(const View<D, P...>& v, std::pair<I, I> r) {
  static_assert(View<D, P...>::rank == 1, "the shim's subview takes index pairs of rank-1 views");
  View<D, P...> s = v;
  s.ptr_ = v.data() + r.first;
  s.ext_[0] = (std::size_t)(r.second - r.first);
  return s;
}
template <class D, class... P, class I, class J>
inline View<D, P...> subview(const View<D, P...>& v, std::pair<I, J> r) {
  return subview(v, std::pair<std::int64_t, std::int64_t>((std::int64_t)r.first, (std::int64_t)r.second));
}

// ---------------------------------------------------------------- parallel --
template <class... Args> struct RangePolicy {
  std::int64_t begin = 0, end = 0;
  RangePolicy(std::int64_t b, std::int64_t e) : begin(b), end(e) {}
  template <class E, class = std::enable_if_t<is_execution_space_v<E>>>
  RangePolicy(const E&, std::int64_t b, std::int64_t e) : begin(b), end(e) {}
};

namespace shim {
template <class... A> inline std::pair<std::int64_t, std::int64_t> range_of(const RangePolicy<A...>& p) {
  return {p.begin, p.end};
}
template <class I, class = std::enable_if_t<std::is_integral_v<I>>>
inline std::pair<std::int64_t, std::int64_t> range_of(I n) {
  return {0, (std::int64_t)n};
}
}  // namespace shim

template <class Policy, class F> inline void parallel_for(const Policy& policy, const F& f) {
  const auto r = shim::range_of(policy);
#pragma omp parallel for schedule(static)
  for (std::int64_t i = r.first; i < r.second; ++i) f(i);
}
template <class Policy, class F>
inline void parallel_for(const std::string&, const Policy& policy, const F& f) {
  parallel_for(policy, f);
}
template <class Policy, class F> inline void parallel_for(const char*, const Policy& policy, const F& f) {
  parallel_for(policy, f);
}

template <class T> struct Sum {
  using value_type = T;
  T& ref;
  explicit Sum(T& r) : ref(r) {}
  static void init(T& v) { v = T(0); }
  static void join(T& a, const T& b) { a += b; }
};

template <class Policy, class F, class T>
inline void parallel_reduce(const Policy& policy, const F& f, const Sum<T>& red) {
  const auto r = shim::range_of(policy);
  T total(0);
#pragma omp parallel
  {
    T local(0);
#pragma omp for schedule(static)
    for (std::int64_t i = r.first; i < r.second; ++i) f(i, local);
#pragma omp critical
    total += local;
  }
  red.ref = total;
}
template <class Policy, class F, class T, class = std::enable_if_t<std::is_arithmetic_v<T>>>
inline void parallel_reduce(const Policy& policy, const F& f, T& result) {
  parallel_reduce(policy, f, Sum<T>(result));
}
template <class Policy, class F, class R>
inline void parallel_reduce(const std::string&, const Policy& policy, const F& f, R&& red) {
  parallel_reduce(policy, f, std::forward<R>(red));
}
template <class Policy, class F, class R>
inline void parallel_reduce(const char*, const Policy& policy, const F& f, R&& red) {
  parallel_reduce(policy, f, std::forward<R>(red));
}

inline void initialize(int = 0, char** = nullptr) {}
inline void finalize() {}
struct ScopeGuard {
  ScopeGuard(int = 0, char** = nullptr) {}
};

}  // namespace Kokkos
