// Parameter updates of a planned model without a re-plan (C ABI part).
//
// After the first forward a model's parameters live in device images laid
// out for its kernel (param_map.h).  Updates go straight to those images:
//  * ponni_b200_set_trainable_parameters (host values; also reached by
//    load_weights) copies the values through a pinned staging buffer and
//    scatters them on the device, stream-ordered after the forwards already
//    queued and without waiting for them;
//  * ponni_b200_set_trainable_parameters_device takes the values from device
//    memory in fp32/fp64/fp16/bf16 and converts them to the model dtype on
//    the device (reference generated set_parameters,
//    src/generator/kokkos_nn/emitter.py:1826-1866); the host copy of the
//    parameters is then read back only when something needs it;
//  * ponni_b200_check_parameters counts image locations that disagree with
//    the packed parameters and trainable values that are not finite
//    (reference parameters_synchronized / parameters_are_finite,
//    emitter.py:1868-1895).
// The model-specialised narrow kernel takes its parameters as a kernel
// argument, so an update from device memory of such a model reads the
// packed parameters back (at most 32 KB) and waits for it.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "model.h"

using namespace ponni_b200;

namespace {

ponni_b200_status cfail(ponni_b200_model* m, cudaError_t e, const char* what) {
  return pb_fail(m, PONNI_B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int dtype_code(ponni_b200_dtype t) {
  switch (t) {
    case PONNI_B200_F32: return 0;
    case PONNI_B200_F64: return 1;
    case PONNI_B200_F16: return 2;
    default: return 3;
  }
}

bool valid_dtype(int t) {
  return t == PONNI_B200_F32 || t == PONNI_B200_F64 || t == PONNI_B200_F16 || t == PONNI_B200_BF16;
}

void images_of(const ponni_b200_model* m, void* img[PIMG_COUNT]) {
  img[PIMG_PACKED] = m->packed_dev;
  img[PIMG_TC] = m->kernel == 2 ? m->tc_image_dev : nullptr;
  img[PIMG_TS] = (m->kernel == 5 || m->kernel == 6) ? m->ts_image_dev : nullptr;
}

// Element copies between tuple order and packed positions (esz 2, 4 or 8).
template <class W>
void gather_packed(W* dst, const W* packed, const uint32_t* packed_of, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = packed[packed_of[i]];
}
template <class W>
void scatter_packed(W* packed, const W* src, const uint32_t* packed_of, int64_t n) {
  for (int64_t i = 0; i < n; ++i) packed[packed_of[i]] = src[i];
}

// The layers' canonical arrays from the packed image (host copy).  Needs the
// uploaded map.
void unpack_to_layers(ponni_b200_model* m, const unsigned char* packed) {
  const size_t esz = m->pmap.esz;
  const uint32_t* po = m->pmap_dev.packed_of_host.data();
  for (const ParamMap::Range& r : m->pmap.ranges) {
    unsigned char* dst = const_cast<unsigned char*>(r.begin);
    const int64_t n = (int64_t)((r.end - r.begin) / (ptrdiff_t)esz);
    if (esz == 8) gather_packed((uint64_t*)dst, (const uint64_t*)packed, po + r.base, n);
    else if (esz == 4) gather_packed((uint32_t*)dst, (const uint32_t*)packed, po + r.base, n);
    else gather_packed((uint16_t*)dst, (const uint16_t*)packed, po + r.base, n);
  }
}

void free_map(ParamMapDev& d, bool all) {
  if (d.recs) cudaFree(d.recs);
  if (d.packed_of) cudaFree(d.packed_of);
  if (d.counts) cudaFree(d.counts);
  d.recs = nullptr;
  d.packed_of = nullptr;
  d.counts = nullptr;
  d.n_recs = d.n_trainable = 0;
  if (all) {
    if (d.pinned_free) cudaEventSynchronize(d.pinned_free);
    if (d.staging) cudaFree(d.staging);
    if (d.pinned) cudaFreeHost(d.pinned);
    if (d.pinned_free) cudaEventDestroy(d.pinned_free);
    if (d.done) cudaEventDestroy(d.done);
    d.staging = d.pinned = nullptr;
    d.pinned_free = d.done = nullptr;
    d.staging_bytes = 0;
  }
}

// Upload the current plan's map (the first update after a plan).
ponni_b200_status upload_map(ponni_b200_model* m) {
  if (m->pmap_uploaded) return PONNI_B200_OK;
  if (m->pmap.overflow)
    return pb_fail(m, PONNI_B200_ERR_UNSUPPORTED, "parameter images exceed 32-bit offsets; device updates unavailable");
  const int64_t nt = ponni_b200_num_trainable_parameters(m);
  std::vector<ParamRec> recs = m->pmap.recs;
  std::sort(recs.begin(), recs.end(), [](const ParamRec& a, const ParamRec& b) {
    return a.img != b.img ? a.img < b.img : a.dst < b.dst;
  });
  std::vector<uint32_t> packed_of((size_t)std::max<int64_t>(nt, 1), 0xffffffffu);
  for (const ParamRec& r : recs) {
    if (r.img != PIMG_PACKED) continue;
    if ((int64_t)r.src >= nt || packed_of[r.src] != 0xffffffffu)
      return pb_fail(m, PONNI_B200_ERR_UNSUPPORTED, "internal: parameter map is not one-to-one");
    packed_of[r.src] = (uint32_t)(r.dst / m->pmap.esz);
  }
  for (int64_t i = 0; i < nt; ++i)
    if (packed_of[i] == 0xffffffffu)
      return pb_fail(m, PONNI_B200_ERR_UNSUPPORTED, "internal: a trainable parameter has no packed location");
  DeviceGuard g(m->device);
  ParamMapDev& d = m->pmap_dev;
  cudaStreamSynchronize(m->stream);
  free_map(d, false);
  cudaError_t e = cudaMalloc(&d.recs, std::max<size_t>(recs.size(), 1) * sizeof(ParamRec));
  if (e == cudaSuccess) e = cudaMalloc(&d.packed_of, packed_of.size() * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&d.counts, 2 * sizeof(int));
  if (e == cudaSuccess && !recs.empty())
    e = cudaMemcpy(d.recs, recs.data(), recs.size() * sizeof(ParamRec), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(d.packed_of, packed_of.data(), packed_of.size() * sizeof(uint32_t), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    free_map(d, false);
    return cfail(m, e, "parameter map upload");
  }
  d.n_recs = (int64_t)recs.size();
  d.n_trainable = nt;
  d.packed_of_host.swap(packed_of);
  m->pmap_uploaded = true;
  return PONNI_B200_OK;
}

// Plan if needed and make the map resident.
ponni_b200_status prepare(ponni_b200_model* m) {
  DeviceGuard g(m->device);
  ponni_b200_status st = pb_plan(m);
  if (st) return st;
  return upload_map(m);
}

// Order the model stream after work queued on `s`.
ponni_b200_status join_model_stream(ponni_b200_model* m, cudaStream_t s) {
  if (s == m->stream) return PONNI_B200_OK;
  ParamMapDev& d = m->pmap_dev;
  cudaError_t e = cudaSuccess;
  if (!d.done) e = cudaEventCreateWithFlags(&d.done, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventRecord(d.done, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(m->stream, d.done, 0);
  return e == cudaSuccess ? PONNI_B200_OK : cfail(m, e, "stream ordering");
}

// After a scatter on the model stream: the specialised narrow kernel needs
// its argument block re-derived from the packed parameters on the host.
ponni_b200_status refresh_host_after_device_update(ponni_b200_model* m) {
  if (m->kernel != 4) {
    m->host_params_stale = true;
    return PONNI_B200_OK;
  }
  cudaError_t e = cudaMemcpyAsync(m->packed_host.data(), m->packed_dev, m->packed_host.size(), cudaMemcpyDeviceToHost,
                                  m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return cfail(m, e, "parameter read-back");
  narrow_jit_refresh((int)m->dtype, m->prog, m->packed_host, &m->jit);
  unpack_to_layers(m, m->packed_host.data());
  m->host_params_stale = false;
  return PONNI_B200_OK;
}

}  // namespace

void pb_free_param_map(ponni_b200_model* m) { free_map(m->pmap_dev, true); }

// Read device-updated parameters back into the layers and packed_host.
ponni_b200_status pb_pull_params(ponni_b200_model* m) {
  if (!m->host_params_stale) return PONNI_B200_OK;
  DeviceGuard g(m->device);
  cudaError_t e = cudaMemcpyAsync(m->packed_host.data(), m->packed_dev, m->packed_host.size(), cudaMemcpyDeviceToHost,
                                  m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return cfail(m, e, "parameter read-back");
  unpack_to_layers(m, m->packed_host.data());
  m->host_params_stale = false;
  return PONNI_B200_OK;
}

// Host values (model dtype, tuple order; already copied into the layers)
// into the device images of a planned model.  Non-OK: the caller re-plans.
ponni_b200_status pb_update_params_from_host(ponni_b200_model* m, const void* host, int64_t n) {
  if (const char* env = getenv("PONNI_B200_PARAM_SCATTER"))
    if (env[0] == '0') return PONNI_B200_ERR_UNSUPPORTED;
  if (!m->planned || m->params_dirty) return PONNI_B200_ERR_UNSUPPORTED;
  ponni_b200_status st = upload_map(m);
  if (st) return st;
  DeviceGuard g(m->device);
  ParamMapDev& d = m->pmap_dev;
  const size_t esz = m->pmap.esz;
  const size_t bytes = std::max<size_t>((size_t)n * esz, 16);
  cudaError_t e = cudaSuccess;
  if (!d.pinned_free) e = cudaEventCreateWithFlags(&d.pinned_free, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventSynchronize(d.pinned_free);  // the previous copy has left the pinned buffer
  if (e == cudaSuccess && bytes > d.staging_bytes) {
    cudaStreamSynchronize(m->stream);
    if (d.staging) cudaFree(d.staging);
    if (d.pinned) cudaFreeHost(d.pinned);
    d.staging = d.pinned = nullptr;
    d.staging_bytes = 0;
    e = cudaMalloc(&d.staging, bytes);
    if (e == cudaSuccess) e = cudaMallocHost(&d.pinned, bytes);
    if (e == cudaSuccess) d.staging_bytes = bytes;
  }
  if (e != cudaSuccess) return cfail(m, e, "parameter staging");
  memcpy(d.pinned, host, (size_t)n * esz);
  e = cudaMemcpyAsync(d.staging, d.pinned, (size_t)n * esz, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaEventRecord(d.pinned_free, m->stream);
  void* img[PIMG_COUNT];
  images_of(m, img);
  if (e == cudaSuccess) e = launch_param_scatter(d, d.staging, dtype_code(m->dtype), dtype_code(m->dtype), img, m->stream);
  if (e != cudaSuccess) return cfail(m, e, "parameter scatter");
  // The host mirror of the packed image follows the same map.
  const uint32_t* po = d.packed_of_host.data();
  unsigned char* ph = m->packed_host.data();
  if (esz == 8) scatter_packed((uint64_t*)ph, (const uint64_t*)host, po, n);
  else if (esz == 4) scatter_packed((uint32_t*)ph, (const uint32_t*)host, po, n);
  else scatter_packed((uint16_t*)ph, (const uint16_t*)host, po, n);
  if (m->kernel == 4) narrow_jit_refresh((int)m->dtype, m->prog, m->packed_host, &m->jit);
  return PONNI_B200_OK;
}

extern "C" {

ponni_b200_status ponni_b200_set_trainable_parameters_device(ponni_b200_model* m, const void* src,
                                                              ponni_b200_dtype src_dtype, int64_t count,
                                                              void* stream) {
  if (!m || !valid_dtype(src_dtype)) return PONNI_B200_ERR_INVALID_ARGUMENT;
  const int64_t need = ponni_b200_num_trainable_parameters(m);
  if (count < need) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "ERROR: trainable input too small");
  if (need > 0 && !src) return PONNI_B200_ERR_INVALID_ARGUMENT;
  ponni_b200_status st = prepare(m);
  if (st) return st;
  if (need == 0) return PONNI_B200_OK;
  DeviceGuard g(m->device);
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  void* img[PIMG_COUNT];
  images_of(m, img);
  cudaError_t e = launch_param_scatter(m->pmap_dev, src, dtype_code(src_dtype), dtype_code(m->dtype), img, s);
  if (e != cudaSuccess) return cfail(m, e, "parameter scatter");
  st = join_model_stream(m, s);
  if (st) return st;
  return refresh_host_after_device_update(m);
}

ponni_b200_status ponni_b200_get_trainable_parameters_device(ponni_b200_model* m, void* dst,
                                                              ponni_b200_dtype dst_dtype, int64_t count,
                                                              void* stream) {
  if (!m || !valid_dtype(dst_dtype)) return PONNI_B200_ERR_INVALID_ARGUMENT;
  const int64_t need = ponni_b200_num_trainable_parameters(m);
  if (count < need) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "output buffer too small");
  if (need > 0 && !dst) return PONNI_B200_ERR_INVALID_ARGUMENT;
  ponni_b200_status st = prepare(m);
  if (st) return st;
  if (need == 0) return PONNI_B200_OK;
  DeviceGuard g(m->device);
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  if (s != m->stream) {  // after updates queued on the model stream
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ev, m->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ev, 0);
    cudaEventDestroy(ev);
    if (e != cudaSuccess) return cfail(m, e, "stream ordering");
  }
  cudaError_t e = launch_param_gather(m->pmap_dev, m->packed_dev, dst, dtype_code(dst_dtype), dtype_code(m->dtype), s);
  return e == cudaSuccess ? PONNI_B200_OK : cfail(m, e, "parameter gather");
}

ponni_b200_status ponni_b200_check_parameters(ponni_b200_model* m, int64_t* mismatches, int64_t* nonfinite) {
  if (!m) return PONNI_B200_ERR_INVALID_ARGUMENT;
  ponni_b200_status st = prepare(m);
  if (st) return st;
  DeviceGuard g(m->device);
  void* img[PIMG_COUNT];
  images_of(m, img);
  int counts[2] = {0, 0};
  cudaError_t e = launch_param_check(m->pmap_dev, dtype_code(m->dtype), img, m->stream);
  if (e == cudaSuccess && m->pmap_dev.counts)
    e = cudaMemcpyAsync(counts, m->pmap_dev.counts, sizeof counts, cudaMemcpyDeviceToHost, m->stream);
  std::vector<unsigned char> packed(m->packed_host.size());
  if (e == cudaSuccess && m->kernel == 4)
    e = cudaMemcpyAsync(packed.data(), m->packed_dev, packed.size(), cudaMemcpyDeviceToHost, m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return cfail(m, e, "parameter check");
  int64_t mism = counts[0];
  if (m->kernel == 4) {  // the specialised kernel's argument block
    NarrowJit want;
    narrow_jit_refresh((int)m->dtype, m->prog, packed, &want);
    const size_t n = std::max(m->prog.n_params, 1);
    const size_t eb = want.params.size() / n;
    if (want.params.size() != m->jit.params.size()) {
      mism += (int64_t)n;
    } else {
      for (size_t i = 0; i < n; ++i)
        if (memcmp(want.params.data() + i * eb, m->jit.params.data() + i * eb, eb) != 0) ++mism;
    }
  }
  if (mismatches) *mismatches = mism;
  if (nonfinite) *nonfinite = counts[1];
  return PONNI_B200_OK;
}

}  // extern "C"
