// Internal model object behind the libponni_b200 C ABI.
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "../../include/ponni_b200.h"
#include "program.h"
#include "narrow_jit.h"
#include "narrow_kernel.h"
#include "param_map.h"
#include "tc_program.h"
#include "tc_resid.h"
#include "tc_stream.h"

namespace ponni_b200 {

struct Layer {
  ponni_b200_layer_desc d;            // params pointer cleared; data lives in `params`
  double raw_scalar[3] = {0, 0, 0};   // the scalars as given (d.scalar is rounded to the model dtype)
  std::vector<unsigned char> params;  // canonical parameters, model dtype
  int64_t num_params() const;         // all parameters the layer owns (elements)
  int64_t num_trainable() const;      // reference get_num_trainable_parameters()
};

size_t dtype_bytes(ponni_b200_dtype t);
double round_to_dtype(ponni_b200_dtype t, double v);
double load_scalar(ponni_b200_dtype t, const unsigned char* p);
void store_scalar(ponni_b200_dtype t, unsigned char* p, double v);
const char* layer_label(int kind);
bool is_dense(int kind);
bool is_pointwise(int kind);
bool overwrites_input(int kind);
bool is_save(int kind);
bool is_binop(int kind);

}  // namespace ponni_b200

struct ponni_b200_model {
  ponni_b200_dtype dtype;
  int device = 0;
  cudaStream_t stream = nullptr;       // current stream (own or user-set)
  cudaStream_t own_stream = nullptr;
  cudaStream_t copy_stream = nullptr;  // second stream of forward_host
  std::vector<ponni_b200::Layer> layers;
  std::string last_error;

  // Execution plan (built lazily on the first forward after a change).
  bool planned = false;
  bool params_dirty = true;
  ponni_b200::Program prog;
  size_t smem_bytes = 0;
  int grid = 0;
  std::vector<unsigned char> packed_host;  // packed parameters (model dtype)
  void* packed_dev = nullptr;
  size_t packed_dev_bytes = 0;
  int num_sms = 0;

  // Tensor-core dense-chain kernel (planned when eligible and allowed).
  int arithmetic = PONNI_B200_ARITH_AUTO;  // ponni_b200_arithmetic requested
  int kernel = 0;       // 1 tile (SIMT), 2 tensor-core, 3 narrow streaming kernel, 4 its model-specialised
                        // (NVRTC-compiled) form, 5 tensor-core kernel with streamed weights,
                        // 6 tensor-core kernel for LayerNorm / residual chains (fp32 split);
                        // 0 = not planned yet
  int narrow_maxw = 0;
  ponni_b200::NarrowLaunch narrow;     // narrow kernel launch configuration
  void* prog_dev = nullptr;            // the Program in device memory (narrow kernel)
  ponni_b200::NarrowJit jit;           // model-specialised narrow kernel (kernel 4)
  std::string jit_why;                 // why the specialised kernel is not used
  ponni_b200::TcProgram tcp;
  void* tc_image_dev = nullptr;
  size_t tc_image_bytes = 0;
  int tc_grid = 0;
  ponni_b200::TsProgram tsp;            // streamed-weights tensor-core kernel (kernel 5)
  void* ts_image_dev = nullptr;
  size_t ts_image_bytes = 0;             // (also the image of kernel 6)
  ponni_b200::TrProgram trp;            // LayerNorm / residual tensor-core kernel (kernel 6)
  void* scratch_dev = nullptr;          // its saved-state scratch (num_sms x scratch_per_cta)
  size_t scratch_bytes = 0;
  int* err_dev = nullptr;  // device error word (bounded waits that gave up)
  std::string tc_why;      // why the tensor-core kernel is not used
  const void* tc_jit = nullptr;  // model-specialised build of the tensor-core kernel 2 or 5 (NVRTC)
  std::string tc_jit_why;        // why it is not used

  int64_t capacity = 0;  // reference internal_state_capacity()
  void* stage_dev = nullptr;  // forward_host staging buffers
  size_t stage_bytes = 0;
  // Device-side parameter updates: where each trainable parameter lives in
  // the planned images (rebuilt by every plan) and its device copy.
  ponni_b200::ParamMap pmap;
  ponni_b200::ParamMapDev pmap_dev;
  bool pmap_uploaded = false;
  // The device images hold newer parameters than `layers[].params` and
  // `packed_host` (after an update from device memory); read back on demand.
  bool host_params_stale = false;
};

namespace ponni_b200 {
// Makes `device` current for the lifetime of the guard and restores the
// caller's current device afterwards: every C-ABI entry point that touches
// the GPU holds one, so a multi-GPU application's current device never
// changes under it.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      cudaGetLastError();
      prev = -1;
    }
    if (prev != device && cudaSetDevice(device) != cudaSuccess) cudaGetLastError();
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
};
}  // namespace ponni_b200

// Helpers shared by the C ABI translation units.
ponni_b200_status pb_fail(ponni_b200_model* m, ponni_b200_status s, const std::string& msg);
ponni_b200_status pb_validate(ponni_b200_model* m);
ponni_b200_status pb_plan(ponni_b200_model* m);
ponni_b200_status pb_ensure_cuda(ponni_b200_model* m);
// After the model's stream has been synchronised: PONNI_B200_ERR_DEVICE (and
// the word cleared) when a kernel recorded a device-side error, else OK.
ponni_b200_status pb_check_device_error(ponni_b200_model* m);
std::string pb_schema_fingerprint(const ponni_b200_model* m);
ponni_b200_status pb_pull_params(ponni_b200_model* m);
ponni_b200_status pb_update_params_from_host(ponni_b200_model* m, const void* host, int64_t n);
void pb_free_param_map(ponni_b200_model* m);
