// Model-specialised kernels compiled at plan time: the narrow-chain kernel
// (source generated from the program, see narrow_jit.h) and the resident
// tensor-core kernel (tc_kernel_body.cuh with the layer structure as
// compile-time constants, see tc_kernel.h).  NVRTC compilation (libnvrtc is
// opened at run time, so the library has no link dependency on it), loading,
// caching and launch.
#include "narrow_jit.h"

#include "tc_kernel.h"
#include "tc_stream.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvrtc.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cstdlib>
#include <vector>
#include <map>
#include <mutex>
#include <sstream>

namespace ponni_b200 {
namespace {

// Texts of the headers the generated kernels include, embedded at build time
// (kJit_<name>).
#include "jit_headers.inc"

constexpr int kJitThreads = 256;
constexpr size_t kMaxParamBytes = 30000;  // kernel parameters are limited to 32764 bytes

// ---- NVRTC, opened at run time ----
struct Nvrtc {
  bool ok = false;
  std::string why;
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetProgramLogSize) log_size = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcGetCUBINSize) cubin_size = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
};

const Nvrtc& nvrtc() {
  static Nvrtc n = [] {
    Nvrtc r;
    void* h = nullptr;
    for (const char* name : {"libnvrtc.so.12", "libnvrtc.so"}) {
      h = dlopen(name, RTLD_NOW | RTLD_LOCAL);
      if (h) break;
    }
    if (!h) {
      r.why = "libnvrtc not found";
      return r;
    }
    r.create = reinterpret_cast<decltype(r.create)>(dlsym(h, "nvrtcCreateProgram"));
    r.compile = reinterpret_cast<decltype(r.compile)>(dlsym(h, "nvrtcCompileProgram"));
    r.log_size = reinterpret_cast<decltype(r.log_size)>(dlsym(h, "nvrtcGetProgramLogSize"));
    r.log = reinterpret_cast<decltype(r.log)>(dlsym(h, "nvrtcGetProgramLog"));
    r.cubin_size = reinterpret_cast<decltype(r.cubin_size)>(dlsym(h, "nvrtcGetCUBINSize"));
    r.cubin = reinterpret_cast<decltype(r.cubin)>(dlsym(h, "nvrtcGetCUBIN"));
    r.destroy = reinterpret_cast<decltype(r.destroy)>(dlsym(h, "nvrtcDestroyProgram"));
    r.ok = r.create && r.compile && r.log_size && r.log && r.cubin_size && r.cubin && r.destroy;
    if (!r.ok) r.why = "libnvrtc lacks an expected entry point";
    return r;
  }();
  return n;
}

// ---- source generation ----
int elem_bytes(int dtype) { return dtype == 1 ? 8 : dtype == 0 ? 4 : 2; }
int compute_bytes(int dtype) { return dtype == 1 ? 8 : 4; }

// Exact literal of a compute-type value (bit pattern, so nothing is lost).
std::string lit(int dtype, double v) {
  char buf[64];
  if (dtype == 1) {
    unsigned long long u;
    memcpy(&u, &v, 8);
    snprintf(buf, sizeof buf, "__longlong_as_double(0x%016llxLL)", u);
  } else {
    const float f = (float)v;
    unsigned u;
    memcpy(&u, &f, 4);
    snprintf(buf, sizeof buf, "__int_as_float(0x%08x)", u);
  }
  return buf;
}

const char* prelude(int dtype) {
  switch (dtype) {
    case 0:
      return "typedef float C;\ntypedef float S;\n"
             "__device__ __forceinline__ C LD(S v) { return v; }\n"
             "__device__ __forceinline__ S ST(C v) { return v; }\n"
             "__device__ __forceinline__ C R(C v) { return v; }\n"
             "__device__ __forceinline__ C FMA(C a, C b, C c) { return fmaf(a, b, c); }\n";
    case 1:
      return "typedef double C;\ntypedef double S;\n"
             "__device__ __forceinline__ C LD(S v) { return v; }\n"
             "__device__ __forceinline__ S ST(C v) { return v; }\n"
             "__device__ __forceinline__ C R(C v) { return v; }\n"
             "__device__ __forceinline__ C FMA(C a, C b, C c) { return fma(a, b, c); }\n";
    case 2:
      return "typedef float C;\ntypedef unsigned short S;\n"
             "__device__ __forceinline__ C LD(S v) { float f; asm(\"cvt.f32.f16 %0, %1;\" : \"=f\"(f) : \"h\"(v)); "
             "return f; }\n"
             "__device__ __forceinline__ S ST(C v) { unsigned short h; asm(\"cvt.rn.f16.f32 %0, %1;\" : \"=h\"(h) : "
             "\"f\"(v)); return h; }\n"
             "__device__ __forceinline__ C R(C v) { return LD(ST(v)); }\n";
    default:
      return "typedef float C;\ntypedef unsigned short S;\n"
             "__device__ __forceinline__ C LD(S v) { return __uint_as_float(((unsigned)v) << 16); }\n"
             "__device__ __forceinline__ S ST(C v) { unsigned short h; asm(\"cvt.rn.bf16.f32 %0, %1;\" : \"=h\"(h) : "
             "\"f\"(v)); return h; }\n"
             "__device__ __forceinline__ C R(C v) { return LD(ST(v)); }\n";
  }
}

// Columns per thread: up to two 16-byte vectors of each input row, capped so
// that a state array holds at most 64 (fp64: 32) values.
int jit_cols(int dtype, int maxw) {
  const int vec = 16 / elem_bytes(dtype);
  const int cap = std::max((dtype == 1 ? 32 : 64) / std::max(maxw, 1), dtype == 1 ? 1 : 2);
  int v = std::min(2 * vec, cap), p2 = 1;
  while (p2 * 2 <= v) p2 *= 2;
  return p2;
}

// One epilogue entry applied to `acc` for feature index variable `f`.
void emit_epi(std::ostringstream& o, int dtype, const EpiDesc& d, const char* f) {
  switch (d.kind) {
    case EPI_BIAS: o << "        acc = R(acc + P.w[" << d.p_off << " + " << f << "]);\n"; break;
    case EPI_RELU: o << "        acc = acc > C(0) ? acc : C(0);\n"; break;
    case EPI_LEAKY_RELU: o << "        acc = R(acc > C(0) ? acc : " << lit(dtype, d.s0) << " * acc);\n"; break;
    default:
      if ((dtype == 2 || dtype == 3) && (d.flags & EPI_FLAG_REF16))  // fp16 / bf16
        o << "        acc = R(ponni_b200::activation16(" << d.kind << ", " << d.flags << ", acc, " << lit(dtype, d.s0)
          << ", " << lit(dtype, d.s1) << ", [](float x) { return R(x); }));\n";
      else
        o << "        acc = R(ponni_b200::activation<C>(" << d.kind << ", " << d.flags << ", acc, " << lit(dtype, d.s0)
          << ", " << lit(dtype, d.s1) << "));\n";
  }
}

}  // namespace

std::string narrow_jit_source(int dtype, const Program& p, int maxw, int* cols_out) {
  const int V = jit_cols(dtype, maxw);
  const int es = elem_bytes(dtype);
  const int VN = std::min(V, 16 / es);  // elements per vector access
  const int NV = V / VN;
  const char* vt = VN * es == 16 ? "uint4" : VN * es == 8 ? "uint2" : VN * es == 4 ? "unsigned int" : "unsigned short";
  if (cols_out) *cols_out = V;
  std::ostringstream o;
  o << "// generated: narrow chain, dtype " << dtype << ", " << p.n_steps << " steps\n";
  o << "#include \"activation.cuh\"\n" << prelude(dtype);
  o << "struct Params { C w[" << std::max(p.n_params, 1) << "]; };\n";
  o << "#define V " << V << "\n";
  o << "extern \"C\" __global__ void __launch_bounds__(" << kJitThreads << ")\n"
    << "ponni_narrow_jit(const __grid_constant__ Params P, const S* __restrict__ in, long long in_ld,\n"
    << "                 S* __restrict__ out, long long out_ld, long long batch, int vec_io) {\n"
    << "  const long long ngroups = (batch + V - 1) / V;\n"
    << "  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < ngroups;\n"
    << "       g += (long long)gridDim.x * blockDim.x) {\n"
    << "    const long long col = g * V;\n"
    << "    const bool full = vec_io && col + V <= batch;\n"
    << "    C s0[" << p.nin << "][V];\n"
    << "    if (full) {\n"
    << "#pragma unroll\n"
    << "      for (int f = 0; f < " << p.nin << "; ++f) {\n"
    << "        const S* src = in + f * in_ld + col;\n"
    << "#pragma unroll\n"
    << "        for (int q = 0; q < " << NV << "; ++q) {\n"
    << "          const " << vt << " u = *reinterpret_cast<const " << vt << "*>(src + q * " << VN << ");\n"
    << "          const S* e = reinterpret_cast<const S*>(&u);\n"
    << "#pragma unroll\n"
    << "          for (int j = 0; j < " << VN << "; ++j) s0[f][q * " << VN << " + j] = LD(e[j]);\n"
    << "        }\n"
    << "      }\n"
    << "    } else {\n"
    << "#pragma unroll\n"
    << "      for (int f = 0; f < " << p.nin << "; ++f)\n"
    << "#pragma unroll\n"
    << "        for (int j = 0; j < V; ++j) s0[f][j] = col + j < batch ? LD(in[f * in_ld + col + j]) : C(0);\n"
    << "    }\n";
  int cur = 0, width = p.nin, next = 1;
  for (int si = 0; si < p.n_steps; ++si) {
    const StepDesc& s = p.steps[si];
    if (s.kind == STEP_DENSE) {
      // Reference order per output: acc from 0, k ascending (Matvec::compute_output,
      // src/ponni_Inference.h:416-426), then the fused epilogue (:428-444).
      const int n = next++;
      o << "    C s" << n << "[" << s.nout << "][V];\n"
        << "#pragma unroll\n"
        << "    for (int o = 0; o < " << s.nout << "; ++o) {\n"
        << "#pragma unroll\n"
        << "      for (int j = 0; j < V; ++j) {\n";
      if (dtype <= 1) {
        o << "        C acc = FMA(P.w[" << s.w_off << " + o], s" << cur << "[0][j], C(0));\n"
          << "#pragma unroll\n"
          << "        for (int k = 1; k < " << s.nin << "; ++k) acc = FMA(P.w[" << s.w_off << " + k * " << s.nout_pad
          << " + o], s" << cur << "[k][j], acc);\n";
      } else {
        o << "        C acc = R(C(0) + R(P.w[" << s.w_off << " + o] * s" << cur << "[0][j]));\n"
          << "#pragma unroll\n"
          << "        for (int k = 1; k < " << s.nin << "; ++k) acc = R(acc + R(P.w[" << s.w_off << " + k * "
          << s.nout_pad << " + o] * s" << cur << "[k][j]));\n";
      }
      for (int e = s.epi_first; e < s.epi_first + s.n_epi; ++e) emit_epi(o, dtype, p.epi[e], "o");
      o << "        s" << n << "[o][j] = acc;\n"
        << "      }\n"
        << "    }\n";
      cur = n;
      width = s.nout;
    } else {  // a pointwise run that follows no dense layer, in place
      o << "#pragma unroll\n"
        << "    for (int f = 0; f < " << width << "; ++f) {\n"
        << "#pragma unroll\n"
        << "      for (int j = 0; j < V; ++j) {\n"
        << "        C acc = s" << cur << "[f][j];\n";
      for (int e = s.epi_first; e < s.epi_first + s.n_epi; ++e) emit_epi(o, dtype, p.epi[e], "f");
      o << "        s" << cur << "[f][j] = acc;\n"
        << "      }\n"
        << "    }\n";
    }
  }
  o << "    if (full) {\n"
    << "#pragma unroll\n"
    << "      for (int f = 0; f < " << p.nout << "; ++f) {\n"
    << "        S* dst = out + f * out_ld + col;\n"
    << "#pragma unroll\n"
    << "        for (int q = 0; q < " << NV << "; ++q) {\n"
    << "          " << vt << " u;\n"
    << "          S* e = reinterpret_cast<S*>(&u);\n"
    << "#pragma unroll\n"
    << "          for (int j = 0; j < " << VN << "; ++j) e[j] = ST(s" << cur << "[f][q * " << VN << " + j]);\n"
    << "          *reinterpret_cast<" << vt << "*>(dst + q * " << VN << ") = u;\n"
    << "        }\n"
    << "      }\n"
    << "    } else {\n"
    << "#pragma unroll\n"
    << "      for (int f = 0; f < " << p.nout << "; ++f)\n"
    << "#pragma unroll\n"
    << "        for (int j = 0; j < V; ++j)\n"
    << "          if (col + j < batch) out[f * out_ld + col + j] = ST(s" << cur << "[f][j]);\n"
    << "    }\n"
    << "  }\n"
    << "}\n";
  return o.str();
}

namespace {

struct CacheEntry {
  cudaLibrary_t lib = nullptr;
  cudaKernel_t kernel = nullptr;
};

std::mutex g_cache_mu;
std::map<std::string, CacheEntry>& cache() {
  static std::map<std::string, CacheEntry> c;
  return c;
}

// Headers the generated sources may include: this library's device headers
// and stand-ins for the two host headers they name (the CUDA type headers
// cuda_fp16.h / cuda_bf16.h come from the toolkit's include directory).
const char kJitStdint[] =
    "#pragma once\n"
    "typedef signed char int8_t; typedef short int16_t; typedef int int32_t; typedef long long int64_t;\n"
    "typedef unsigned char uint8_t; typedef unsigned short uint16_t; typedef unsigned int uint32_t;\n"
    "typedef unsigned long long uint64_t; typedef unsigned long long uintptr_t;\n";
const char kJitCudaRuntime[] = "#pragma once\n";
// The one driver type the kernels use: the tensor-map kernel parameter (the
// driver API's definition: 16 64-bit words, 64-byte aligned).
const char kJitCuda[] =
    "#pragma once\n"
    "typedef struct CUtensorMap_st { alignas(64) unsigned long long opaque[16]; } CUtensorMap;\n";

// The CUDA toolkit's include directory (cuda_fp16.h), or "" when none is found.
std::string cuda_include_dir() {
  std::vector<std::string> cands;
  for (const char* env : {"CUDA_HOME", "CUDA_PATH"})
    if (const char* v = getenv(env)) cands.push_back(std::string(v) + "/include");
  cands.push_back("/usr/local/cuda/include");
  for (const std::string& d : cands) {
    FILE* f = fopen((d + "/cuda_fp16.h").c_str(), "r");
    if (f) {
      fclose(f);
      return d;
    }
  }
  return "";
}

bool compile_and_load(const std::string& src, const char* name, cudaKernel_t* kernel, std::string* why) {
  const Nvrtc& n = nvrtc();
  if (!n.ok) {
    *why = n.why;
    return false;
  }
  const char* hdr_src[] = {kJit_epi_kinds_h,        kJit_activation_cuh,    kJit_program_h,
                           kJit_device_math_cuh,    kJit_tc_program_h,      kJit_f32x2_cuh,
                           kJit_tc_common_cuh,      kJit_tc_kernel_body_cuh, kJit_tc_stream_program_h,
                           kJit_tc_stream_body_cuh, kJitStdint,             kJitCudaRuntime,
                           kJitCuda};
  const char* hdr_name[] = {"epi_kinds.h",        "activation.cuh",    "program.h",     "device_math.cuh",
                            "tc_program.h",       "f32x2.cuh",         "tc_common.cuh", "tc_kernel_body.cuh",
                            "tc_stream_program.h", "tc_stream_body.cuh", "stdint.h",    "cuda_runtime.h",
                            "cuda.h"};
  constexpr int nh = (int)(sizeof(hdr_src) / sizeof(hdr_src[0]));
  nvrtcProgram prog = nullptr;
  if (n.create(&prog, src.c_str(), "ponni_jit.cu", nh, hdr_src, hdr_name) != NVRTC_SUCCESS) {
    *why = "nvrtcCreateProgram failed";
    return false;
  }
  const std::string inc = cuda_include_dir();
  const std::string inc_opt = "-I" + inc;
  std::vector<const char*> opts = {"--gpu-architecture=sm_100a", "-std=c++17", "--fmad=true"};
  if (!inc.empty()) opts.push_back(inc_opt.c_str());
  // PONNI_B200_JIT_LOG=1: print the generated source's resource usage (ptxas)
  const char* logv = getenv("PONNI_B200_JIT_LOG");
  const bool verbose = logv && atoi(logv) != 0;
  if (verbose) opts.push_back("--ptxas-options=-v");
  const nvrtcResult rc = n.compile(prog, (int)opts.size(), opts.data());
  if (verbose) {
    size_t ls = 0;
    n.log_size(prog, &ls);
    std::string log(ls, '\0');
    if (ls) n.log(prog, &log[0]);
    fprintf(stderr, "[ponni_b200 jit] %s: %s\n", name, log.c_str());
  }
  if (rc != NVRTC_SUCCESS) {
    size_t ls = 0;
    n.log_size(prog, &ls);
    std::string log(ls, '\0');
    if (ls) n.log(prog, &log[0]);
    *why = "NVRTC compilation failed: " + log.substr(0, 400);
    n.destroy(&prog);
    return false;
  }
  size_t cs = 0;
  n.cubin_size(prog, &cs);
  std::vector<char> cubin(cs);
  n.cubin(prog, cubin.data());
  n.destroy(&prog);
  cudaLibrary_t lib = nullptr;
  cudaError_t e = cudaLibraryLoadData(&lib, cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0);
  if (e == cudaSuccess) e = cudaLibraryGetKernel(kernel, lib, name);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *why = std::string("loading the compiled kernel failed: ") + cudaGetErrorString(e);
    return false;
  }
  cache()[src] = CacheEntry{lib, *kernel};
  return true;
}

void to_compute(int dtype, const std::vector<unsigned char>& packed, int n, std::vector<unsigned char>* out) {
  out->assign((size_t)std::max(n, 1) * compute_bytes(dtype), 0);
  if (dtype <= 1) {
    memcpy(out->data(), packed.data(), std::min(packed.size(), (size_t)n * elem_bytes(dtype)));
    return;
  }
  float* f = reinterpret_cast<float*>(out->data());
  for (int i = 0; i < n && (size_t)(2 * i + 1) < packed.size(); ++i) {
    uint16_t h;
    memcpy(&h, packed.data() + 2 * i, 2);
    uint32_t bits;
    if (dtype == 3) {
      bits = (uint32_t)h << 16;
    } else {  // IEEE half -> float, exact
      const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
      uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff;
      if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
      } else if (exp != 0) {
        bits = sign | ((exp + 112) << 23) | (man << 13);
      } else if (man == 0) {
        bits = sign;
      } else {  // subnormal: normalise
        int e = -1;
        do {
          ++e;
          man <<= 1;
        } while (!(man & 0x400));
        bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3ff) << 13);
      }
    }
    memcpy(&f[i], &bits, 4);
  }
}

}  // namespace

void narrow_jit_refresh(int dtype, const Program& p, const std::vector<unsigned char>& packed, NarrowJit* J) {
  to_compute(dtype, packed, p.n_params, &J->params);
}

bool narrow_jit_build(int dtype, const Program& p, int maxw, const std::vector<unsigned char>& packed, int num_sms,
                      NarrowJit* J, std::string* why) {
  if ((size_t)std::max(p.n_params, 1) * compute_bytes(dtype) > kMaxParamBytes) {
    *why = "parameters exceed the kernel-parameter space";
    return false;
  }
  int cols = 1;
  const std::string src = narrow_jit_source(dtype, p, maxw, &cols);
  cudaKernel_t kernel = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = cache().find(src);
    if (it != cache().end()) kernel = it->second.kernel;
    else if (!compile_and_load(src, "ponni_narrow_jit", &kernel, why)) return false;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reinterpret_cast<const void*>(kernel), kJitThreads, 0) !=
      cudaSuccess) {
    cudaGetLastError();
    per_sm = 2048 / kJitThreads;
  }
  J->kernel = reinterpret_cast<const void*>(kernel);
  J->cols = cols;
  J->elem = elem_bytes(dtype);
  J->grid = num_sms * std::max(per_sm, 1);
  to_compute(dtype, packed, p.n_params, &J->params);
  return true;
}

cudaError_t narrow_jit_launch(const NarrowJit& J, const void* in, int64_t in_ld, void* out, int64_t out_ld,
                              int64_t batch, cudaStream_t stream) {
  const int64_t es = J.elem;
  int vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
            ((in_ld * es) % 16 == 0) && ((out_ld * es) % 16 == 0);
  const int64_t groups = (batch + J.cols - 1) / J.cols;
  const int grid = (int)std::min<int64_t>((groups + kJitThreads - 1) / kJitThreads, J.grid);
  long long a_in_ld = in_ld, a_out_ld = out_ld, a_batch = batch;
  void* args[] = {const_cast<unsigned char*>(J.params.data()), &in, &a_in_ld, &out, &a_out_ld, &a_batch, &vec};
  return cudaLaunchKernel(J.kernel, dim3(grid), dim3(kJitThreads), args, 0, stream);
}


// ---------------------------------------- resident tensor-core kernel ----

namespace {

std::string tc_jit_source(const TcProgram& p) {
  const char* T = p.dtype == 0 ? "float" : p.dtype == 2 ? "__half" : "__nv_bfloat16";
  const int tps = p.slot_threads;
  const int bound = (tps == 128 && p.dtype != 0) ? kTcMaxThreads : kTcMaxThreads / 2;
  std::ostringstream o;
  auto arr = [&](const char* name, auto get) {
    o << "    constexpr int " << name << "[] = {";
    for (int l = 0; l < p.n_layers; ++l) o << (l ? ", " : "") << get(p.layers[l]);
    o << "};\n";
  };
  o << "// generated: resident tensor-core kernel, dtype " << p.dtype << ", " << p.n_layers << " layers\n"
    << "#include \"tc_kernel_body.cuh\"\n"
    << "namespace ponni_b200 {\nnamespace tck {\n"
    << "struct JitShape {\n"
    << "  static constexpr bool kStatic = true;\n"
    << "  static constexpr int kNL = " << p.n_layers << ";\n"
    << "  static __device__ __forceinline__ void fix(int l, TcLayer& L) {\n";
  arr("kK", [](const TcLayer& L) { return L.k_pad; });
  arr("kN", [](const TcLayer& L) { return L.n_pad; });
  arr("kOut", [](const TcLayer& L) { return L.nout; });
  arr("kG", [](const TcLayer& L) { return L.groups; });
  arr("kGS", [](const TcLayer& L) { return L.group_steps; });
  arr("kAct", [](const TcLayer& L) { return L.act; });
  arr("kFl", [](const TcLayer& L) { return L.act_flags; });
  arr("kB", [](const TcLayer& L) { return L.has_bias; });
  arr("kBM", [](const TcLayer& L) { return L.bias_mma; });
  o << "    L.k_pad = kK[l]; L.n_pad = kN[l]; L.nout = kOut[l]; L.groups = kG[l]; L.group_steps = kGS[l];\n"
    << "    L.act = kAct[l]; L.act_flags = kFl[l]; L.has_bias = kB[l]; L.bias_mma = kBM[l];\n"
    << "  }\n};\n}  // namespace tck\n}  // namespace ponni_b200\n"
    << "extern \"C\" __global__ void __launch_bounds__(" << bound << ", 1)\n"
    << "ponni_tc_jit(const __grid_constant__ ponni_b200::TcProgram p, const unsigned char* __restrict__ image,\n"
    << "             const " << T << "* __restrict__ in, long long in_ld, " << T << "* __restrict__ out,\n"
    << "             long long out_ld, long long batch, int in_vec, int* __restrict__ err) {\n"
    << "  ponni_b200::tck::tc_forward_body<" << T << ", " << tps << ", ponni_b200::tck::JitShape>(\n"
    << "      p, image, in, in_ld, out, out_ld, batch, in_vec, err);\n"
    << "}\n";
  return o.str();
}

}  // namespace

bool tc_jit_build(const TcProgram& p, const void** kernel, std::string* why) {
  if (const char* v = getenv("PONNI_B200_TC_JIT"))
    if (atoi(v) == 0) {
      *why = "disabled (PONNI_B200_TC_JIT=0)";
      return false;
    }
  const std::string src = tc_jit_source(p);
  cudaKernel_t k = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = cache().find(src);
    if (it != cache().end()) k = it->second.kernel;
    else if (!compile_and_load(src, "ponni_tc_jit", &k, why)) return false;
  }
  *kernel = reinterpret_cast<const void*>(k);
  return true;
}

cudaError_t launch_tc_forward_jit(const void* kernel, const TcProgram& p, const void* image, const void* in,
                                  int64_t in_ld, void* out, int64_t out_ld, int64_t batch, int grid, int* err,
                                  cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
  if (e != cudaSuccess) return e;
  const int64_t es = p.dtype == 0 ? 4 : 2;
  int vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && ((in_ld * es) % 16 == 0);
  long long a_in_ld = in_ld, a_out_ld = out_ld, a_batch = batch;
  TcProgram prog = p;
  void* args[] = {&prog, const_cast<void**>(&image), const_cast<void**>(&in), &a_in_ld, &out, &a_out_ld, &a_batch, &vec, &err};
  return cudaLaunchKernel(kernel, dim3(grid), dim3(p.slots * p.slot_threads), args, p.smem_bytes, stream);
}



// ------------------------------------------- streamed tensor-core kernel ----

namespace {

std::string ts_jit_source(const TsProgram& p) {
  const char* T = p.dtype == 2 ? "__half" : "__nv_bfloat16";
  std::ostringstream o;
  o << "// generated: streamed tensor-core kernel, dtype " << p.dtype << ", " << p.n_layers << " layers\n"
    << "#include \"tc_stream_body.cuh\"\n"
    << "namespace ponni_b200 {\nnamespace tsk {\n"
    << "struct TsJitShape {\n"
    << "  static constexpr bool kStatic = true;\n"
    << "  static constexpr int kNL = " << p.n_layers << ";\n";
  // the MMA issuer's per-layer loop bounds
  o << "  static __device__ __forceinline__ void fix(int l, TsLayer& L) {\n    switch (l) {\n";
  for (int l = 0; l < p.n_layers; ++l)
    o << "      case " << l << ": L.k_pad = " << p.layers[l].k_pad << "; L.kblk = " << p.layers[l].kblk
      << "; L.n_pad = " << p.layers[l].n_pad << "; break;\n";
  o << "      default: break;\n    }\n  }\n"
    << "  template <class T>\n"
    << "  static __device__ __forceinline__ void epilogue(int l, const TsLayer& Lr, int, bool last, uint32_t tmem_row,\n"
    << "      int c_begin, const float* bias, uint32_t a_out, T* __restrict__ out, int64_t out_ld, int64_t col,\n"
    << "      int64_t batch, int m, long long (&t_ph)[3]) {\n"
    << "    TsLayer L = Lr;\n"
    << "    switch (l) {\n";
  for (int l = 0; l < p.n_layers; ++l) {
    const TsLayer& L = p.layers[l];
    int act = L.act;  // the activations the streamed epilogue instantiates (others run as none, as its dispatch)
    if (act != EPI_RELU && act != EPI_LEAKY_RELU && act != EPI_SILU && act != EPI_GELU && act != EPI_TANH &&
        act != EPI_SIGMOID)
      act = EPI_NONE;
    o << "      case " << l << ":\n"
      << "        L.n_pad = " << L.n_pad << "; L.nout = " << L.nout << "; L.has_bias = " << L.has_bias
      << "; L.act_flags = " << L.act_flags << ";\n"
      << "        ts_epilogue<T, " << act << ">(L, " << p.fast_act
      << ", last, tmem_row, c_begin, bias, a_out, out, out_ld, col, batch, m, t_ph);\n"
      << "        break;\n";
  }
  o << "      default: break;\n    }\n  }\n};\n"
    << "}  // namespace tsk\n}  // namespace ponni_b200\n"
    << "extern \"C\" __global__ void __launch_bounds__(" << kTsThreads << ", 1)\n"
    << "ponni_ts_jit(const __grid_constant__ ponni_b200::TsProgram p, const unsigned char* __restrict__ image,\n"
    << "             const " << T << "* __restrict__ in, long long in_ld, " << T << "* __restrict__ out,\n"
    << "             long long out_ld, long long batch, int in_vec, const __grid_constant__ CUtensorMap in_map,\n"
    << "             int in_tma, int* __restrict__ err) {\n"
    << "  ponni_b200::tsk::ts_forward_body<" << T << ", false, ponni_b200::tsk::TsJitShape>(\n"
    << "      p, image, in, in_ld, out, out_ld, batch, in_vec, in_map, in_tma, err);\n"
    << "}\n";
  return o.str();
}

}  // namespace

bool ts_jit_build(const TsProgram& p, const void** kernel, std::string* why) {
  if (const char* v = getenv("PONNI_B200_TC_JIT"))
    if (atoi(v) == 0) {
      *why = "disabled (PONNI_B200_TC_JIT=0)";
      return false;
    }
  if (p.pair) {
    *why = "CTA-pair mode runs the library's kernel";
    return false;
  }
  const std::string src = ts_jit_source(p);
  cudaKernel_t k = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = cache().find(src);
    if (it != cache().end()) k = it->second.kernel;
    else if (!compile_and_load(src, "ponni_ts_jit", &k, why)) return false;
  }
  *kernel = reinterpret_cast<const void*>(k);
  return true;
}

}  // namespace ponni_b200
