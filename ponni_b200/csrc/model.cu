// libponni_b200 C ABI: model construction, validation, planning and forward.
//
// Host side of the reference's ponni::Inference (src/ponni_Inference.h) and
// factory (src/ponni_create_model.h).  The reference's compile-time layer
// tuple arrives here as a flat descriptor list; everything the reference
// decides at compile time (fusion blocks, buffer selection, scratch sizes) is
// decided once per model on the host and handed to the fused tile kernel as a
// Program in kernel-parameter (constant) space.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "model.h"
#include "narrow_kernel.h"
#include "tc_kernel.h"
#include "tc_plan.h"
#include "tile_kernel.h"

using namespace ponni_b200;

namespace ponni_b200 {

size_t dtype_bytes(ponni_b200_dtype t) {
  switch (t) {
    case PONNI_B200_F32: return 4;
    case PONNI_B200_F64: return 8;
    case PONNI_B200_F16: return 2;
    case PONNI_B200_BF16: return 2;
  }
  return 0;
}

double load_scalar(ponni_b200_dtype t, const unsigned char* p) {
  switch (t) {
    case PONNI_B200_F32: { float v; memcpy(&v, p, 4); return v; }
    case PONNI_B200_F64: { double v; memcpy(&v, p, 8); return v; }
    case PONNI_B200_F16: { __half v; memcpy(&v, p, 2); return (double)__half2float(v); }
    case PONNI_B200_BF16: { __nv_bfloat16 v; memcpy(&v, p, 2); return (double)__bfloat162float(v); }
  }
  return 0.0;
}

void store_scalar(ponni_b200_dtype t, unsigned char* p, double v) {
  switch (t) {
    case PONNI_B200_F32: { float f = (float)v; memcpy(p, &f, 4); return; }
    case PONNI_B200_F64: { memcpy(p, &v, 8); return; }
    case PONNI_B200_F16: { __half h = __float2half_rn((float)v); memcpy(p, &h, 2); return; }
    case PONNI_B200_BF16: { __nv_bfloat16 h = __float2bfloat16_rn((float)v); memcpy(p, &h, 2); return; }
  }
}

double round_to_dtype(ponni_b200_dtype t, double v) {
  unsigned char b[8];
  store_scalar(t, b, v);
  return load_scalar(t, b);
}

const char* layer_label(int kind) {
  static const char* names[] = {"Matvec",      "Bias",        "ReLU",       "LeakyReLU",  "ELU",
                                "SELU",        "GELU",        "SiLU",       "Sigmoid",    "Tanh",
                                "Softplus",    "HardSigmoid", "HardSwish",  "Mish",       "LayerNorm",
                                "MinMaxNorm",  "Softmax",     "LogSoftmax", "Save_State", "Binop_Add",
                                "Binop_Concatenate", "Binop_Projection_Add"};
  if (kind < 0 || kind > PONNI_B200_BINOP_PROJECTION_ADD) return "Unknown";
  return names[kind];
}

// LayerTraits fusion kinds (src/ponni_LayerTraits.h:10-38): Matvec is dense,
// Bias and the twelve activations are pointwise, everything else a barrier.
bool is_dense(int k) { return k == PONNI_B200_MATVEC; }
bool is_pointwise(int k) { return k >= PONNI_B200_BIAS && k <= PONNI_B200_MISH; }
bool overwrites_input(int k) { return k != PONNI_B200_MATVEC; }
bool is_save(int k) { return k == PONNI_B200_SAVE_STATE; }
bool is_binop(int k) {
  return k == PONNI_B200_BINOP_ADD || k == PONNI_B200_BINOP_CONCATENATE || k == PONNI_B200_BINOP_PROJECTION_ADD;
}

int64_t Layer::num_params() const {
  switch (d.kind) {
    case PONNI_B200_MATVEC: return (int64_t)d.num_inputs * d.num_outputs;
    case PONNI_B200_BIAS: return d.num_inputs;
    case PONNI_B200_LAYER_NORM: return 2 * (int64_t)d.num_inputs;
    case PONNI_B200_BINOP_PROJECTION_ADD: return (int64_t)d.aux * d.num_inputs + d.num_inputs;
    default: return 0;
  }
}

int64_t Layer::num_trainable() const { return (d.flags & PONNI_B200_FLAG_TRAINABLE) ? num_params() : 0; }

}  // namespace ponni_b200

// ---------------------------------------------------------------------------
static thread_local std::string g_create_error;

ponni_b200_status pb_fail(ponni_b200_model* m, ponni_b200_status s, const std::string& msg) {
  if (m) m->last_error = msg;
  return s;
}

static ponni_b200_status cuda_fail(ponni_b200_model* m, cudaError_t e, const char* what) {
  return pb_fail(m, PONNI_B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Per-layer checks of each reference layer's validate() and the tuple walk of
// Inference::validate (src/ponni_Inference.h:719-737).  Messages follow the
// reference's abort texts.
ponni_b200_status pb_validate(ponni_b200_model* m) {
  const int L = (int)m->layers.size();
  std::vector<int> saved(64, 0);
  for (int i = 0; i < L; ++i) {
    const auto& d = m->layers[i].d;
    const char* label = layer_label(d.kind);
    auto bad = [&](const std::string& msg) { return pb_fail(m, PONNI_B200_ERR_VALIDATION, "ERROR: " + msg); };
    if (d.save_index >= 64) return bad("saved-state index must be < 64");
    switch (d.kind) {
      case PONNI_B200_MATVEC:
        if (d.num_inputs <= 0 || d.num_outputs <= 0) return bad("Matvec weights dimensions must be nonzero");
        break;
      case PONNI_B200_BIAS:
        if (d.num_inputs <= 0) return bad("Bias weights must not be empty");
        if (d.num_outputs != d.num_inputs) return bad("Bias input/output size mismatch");
        break;
      case PONNI_B200_LAYER_NORM:
        if (d.num_inputs <= 0) return bad("LayerNorm params must not be empty");
        if (d.num_outputs != d.num_inputs) return bad("LayerNorm gamma/beta size mismatch");
        if (!(d.scalar[0] > 0.0)) return bad("LayerNorm epsilon must be > 0");
        break;
      case PONNI_B200_SAVE_STATE:
        if (d.num_inputs <= 0) return bad("Save_State num_inputs must be > 0");
        if (d.num_outputs != d.num_inputs) return bad("Save_State input/output size mismatch");
        if (d.save_index < 0) return bad("Save_State requires a save index");
        saved[d.save_index] = d.num_inputs;
        break;
      case PONNI_B200_BINOP_ADD:
        if (d.num_inputs <= 0 || d.num_outputs != d.num_inputs) return bad("Binop_Add invalid input/output size");
        if (d.save_index < 0 || d.num_inputs != saved[d.save_index])
          return bad("Binop_Add: Saved layer num inputs != this layer's num inputs");
        break;
      case PONNI_B200_BINOP_CONCATENATE: {
        int s = d.save_index < 0 ? 0 : saved[d.save_index];
        if (d.num_inputs <= 0 || s <= 0) return bad("Binop_Concatenate input sizes must be > 0");
        if (d.num_outputs != s + d.num_inputs)
          return bad("Binop_Concatenate: this layer's num outputs != this layer's num inputs + saved layer's num inputs");
        break;
      }
      case PONNI_B200_BINOP_PROJECTION_ADD:
        if (d.aux <= 0 || d.num_inputs <= 0) return bad("Binop_Projection_Add weights dimensions must be nonzero");
        if (d.num_outputs != d.num_inputs) return bad("Binop_Projection_Add output size mismatch");
        if (d.save_index < 0 || d.aux != saved[d.save_index])
          return bad("Binop_Projection_Add saved layer size incompatible with projection weights");
        break;
      default:
        if (d.kind < 0 || d.kind > PONNI_B200_BINOP_PROJECTION_ADD) return bad("unknown layer kind");
        if (d.num_inputs <= 0) return bad(std::string(label) + " num_inputs must be > 0");
        if (d.num_outputs != d.num_inputs) return bad(std::string(label) + " input/output size mismatch");
        break;
    }
    if (i + 1 < L && d.num_outputs != m->layers[i + 1].d.num_inputs)
      return bad("This layer's num outputs != next layer's num inputs");
  }
  return PONNI_B200_OK;
}

// ---------------------------------------------------------------------------
// Planner: lower the layer list to a Program of on-chip steps.
//
// The walk mirrors traverse_mixed_batch_parallel (src/ponni_Inference.h:454-555):
// a dense layer plus the pointwise layers that follow it is one fused block
// (fused_dense_block_end, :61-70); the final dense block writes the caller's
// output directly; every other layer is a barrier on the materialised state.
// Where the reference ping-pongs between HBM Views tmp1/tmp2, the plan
// ping-pongs between shared-memory tiles A and B.
namespace {

constexpr int BUF_IN = 0, BUF_IN2 = 1, BUF_A = 2, BUF_B = 3, BUF_SAVED0 = 4;

int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

bool fast_activation(int k) {
  return k == PONNI_B200_RELU || k == PONNI_B200_LEAKY_RELU || k == PONNI_B200_SILU || k == PONNI_B200_GELU ||
         k == PONNI_B200_TANH || k == PONNI_B200_SIGMOID;
}

struct Planner {
  ponni_b200_model* m;
  Program& p;
  std::vector<unsigned char>& packed;
  size_t esz;
  int width[kMaxBuffers] = {0};
  ParamMap* rec = nullptr;  // receives the packed location of every trainable parameter

  // Append `n` parameters (canonical, model dtype) to the packed buffer,
  // 16-element aligned; returns the element offset.
  int64_t append(const unsigned char* src, int64_t n) {
    int64_t off = align_up((int64_t)(packed.size() / esz), 16);
    packed.resize((size_t)(off + n) * esz, 0);
    if (n) memcpy(packed.data() + off * esz, src, (size_t)n * esz);
    if (rec)
      for (int64_t i = 0; i < n; ++i) rec->add(src + i * esz, PIMG_PACKED, PENC_MODEL, (size_t)(off + i) * esz);
    return off;
  }
  // Append W[k][o] (rows of nout) padded to rows of nout_pad with zeros.
  int64_t append_matrix(const unsigned char* src, int nin, int nout, int nout_pad) {
    int64_t off = align_up((int64_t)(packed.size() / esz), 16);
    packed.resize((size_t)(off + (int64_t)nin * nout_pad) * esz, 0);
    for (int k = 0; k < nin; ++k) {
      memcpy(packed.data() + (off + (int64_t)k * nout_pad) * esz, src + (size_t)k * nout * esz, (size_t)nout * esz);
      if (rec)
        for (int o = 0; o < nout; ++o)
          rec->add(src + ((size_t)k * nout + o) * esz, PIMG_PACKED, PENC_MODEL,
                   (size_t)(off + (int64_t)k * nout_pad + o) * esz);
    }
    return off;
  }
  ponni_b200_status fail(const std::string& s) { return pb_fail(m, PONNI_B200_ERR_UNSUPPORTED, s); }
  void use(int buf, int w) { width[buf] = std::max(width[buf], w); }

  StepDesc& new_step(int kind) {
    StepDesc& s = p.steps[p.n_steps++];
    memset(&s, 0, sizeof(s));
    s.kind = kind;
    s.src = s.dst = s.aux = -1;
    s.fast_bias_off = -1;
    return s;
  }

  ponni_b200_status add_epilogue(StepDesc& s, int first_layer, int end_layer) {
    s.epi_first = p.n_epi;
    s.n_epi = 0;
    for (int j = first_layer; j < end_layer; ++j) {
      if (p.n_epi >= kMaxEpilogue) return fail("too many pointwise layers for one program");
      const Layer& L = m->layers[j];
      EpiDesc& e = p.epi[p.n_epi++];
      memset(&e, 0, sizeof(e));
      e.kind = L.d.kind;
      e.flags = L.d.flags;
      if ((m->dtype == PONNI_B200_F16 || m->dtype == PONNI_B200_BF16) && m->arithmetic != PONNI_B200_ARITH_GENERATED &&
          L.d.kind != PONNI_B200_BIAS)
        e.flags |= EPI_FLAG_REF16;
      e.s0 = L.d.scalar[0];
      e.s1 = L.d.scalar[1];
      e.s2 = L.d.scalar[2];
      if (L.d.kind == PONNI_B200_BIAS) e.p_off = append(L.params.data(), L.d.num_inputs);
      s.n_epi++;
    }
    // Fast path: [Bias?][one common activation?].
    int j = 0;
    const EpiDesc* ep = p.epi + s.epi_first;
    if (j < s.n_epi && ep[j].kind == EPI_BIAS) s.fast_bias_off = ep[j++].p_off;
    s.fast_act = EPI_NONE;
    if (j < s.n_epi && fast_activation(ep[j].kind)) {
      s.fast_act = ep[j].kind;
      s.fast_act_flags = ep[j].flags;
      s.s0 = ep[j].s0;
      s.s1 = ep[j].s1;
      ++j;
    }
    if (j == s.n_epi) s.flags |= DENSE_FAST_EPI;
    else s.fast_bias_off = -1;
    return PONNI_B200_OK;
  }

  ponni_b200_status run() {
    memset(&p, 0, sizeof(Program));
    const int L = (int)m->layers.size();
    p.nin = m->layers[0].d.num_inputs;
    p.nout = m->layers[L - 1].d.num_outputs;
    p.in_buf = BUF_IN;
    p.in_buf2 = BUF_IN2;
    p.final_buf = -1;
    use(BUF_IN, p.nin);
    use(BUF_IN2, p.nin);
    int cur = BUF_IN;
    int n_saved_buf = 0;
    auto saved_buf = [&](int idx) {
      n_saved_buf = std::max(n_saved_buf, idx + 1);
      return BUF_SAVED0 + idx;
    };
    auto other = [&](int b) { return b == BUF_A ? BUF_B : BUF_A; };
    bool last_to_global = false;
    int i = 0;
    while (i < L) {
      if (p.n_steps >= kMaxSteps) return fail("too many layers for one program");
      const Layer& Ly = m->layers[i];
      const auto& d = Ly.d;
      if (is_dense(d.kind)) {
        int end = i + 1;
        while (end < L && is_pointwise(m->layers[end].d.kind)) ++end;
        StepDesc& s = new_step(STEP_DENSE);
        s.nin = d.num_inputs;
        s.nout = d.num_outputs;
        s.nout_pad = (int)align_up(d.num_outputs, kTO);
        s.src = cur;
        s.w_off = append_matrix(Ly.params.data(), d.num_inputs, d.num_outputs, s.nout_pad);
        int epi_begin = i + 1;
        if (m->arithmetic == PONNI_B200_ARITH_GENERATED) {
          // Generated-model arithmetic (emitter.py:704-708, :975-983): the sum
          // starts at the bias that follows the Matvec; 16-bit products are
          // accumulated with one fused multiply-add each.
          if (epi_begin < end && m->layers[epi_begin].d.kind == PONNI_B200_BIAS) {
            s.flags |= DENSE_INIT_BIAS;
            s.b_off = append(m->layers[epi_begin].params.data(), d.num_outputs);
            ++epi_begin;
          }
          if (m->dtype == PONNI_B200_F16 || m->dtype == PONNI_B200_BF16) s.flags |= DENSE_HALF_FMA;
        }
        ponni_b200_status st = add_epilogue(s, epi_begin, end);
        if (st) return st;
        if (end == L) {
          s.flags |= DENSE_TO_GLOBAL;
          last_to_global = true;
        } else {
          s.dst = other(cur);
          use(s.dst, s.nout);
          cur = s.dst;
        }
        i = end;
        continue;
      }
      if (is_pointwise(d.kind)) {
        int end = i;
        while (end < L && is_pointwise(m->layers[end].d.kind)) ++end;
        StepDesc& s = new_step(STEP_POINTWISE);
        s.nin = s.nout = d.num_inputs;
        s.src = cur;
        ponni_b200_status st = add_epilogue(s, i, end);
        if (st) return st;
        i = end;
        continue;
      }
      switch (d.kind) {
        case PONNI_B200_LAYER_NORM: {
          StepDesc& s = new_step(STEP_LAYERNORM);
          s.nin = s.nout = d.num_inputs;
          s.src = cur;
          s.s0 = d.scalar[0];
          if (m->arithmetic == PONNI_B200_ARITH_GENERATED) {
            // The generated model's LayerNormalization (emitter.py:867-889):
            // Welford; 16-bit models run it in float with a float epsilon
            // (emitter.py:1161-1191).
            s.flags |= LN_WELFORD;
            if (m->dtype == PONNI_B200_F16 || m->dtype == PONNI_B200_BF16) s.s0 = (double)(float)Ly.raw_scalar[0];
          }
          s.w_off = append(Ly.params.data(), d.num_inputs);
          s.b_off = append(Ly.params.data() + (size_t)d.num_inputs * esz, d.num_inputs);
          break;
        }
        case PONNI_B200_MIN_MAX_NORM:
        case PONNI_B200_SOFTMAX:
        case PONNI_B200_LOG_SOFTMAX: {
          StepDesc& s = new_step(d.kind == PONNI_B200_MIN_MAX_NORM ? STEP_MINMAXNORM
                                 : d.kind == PONNI_B200_SOFTMAX    ? STEP_SOFTMAX
                                                                   : STEP_LOGSOFTMAX);
          s.nin = s.nout = d.num_inputs;
          s.src = cur;
          s.s0 = d.scalar[0];
          s.s1 = d.scalar[1];
          s.s2 = d.scalar[2];
          break;
        }
        case PONNI_B200_SAVE_STATE: {
          StepDesc& s = new_step(STEP_COPY);
          s.nin = s.nout = d.num_inputs;
          s.src = cur;
          s.dst = saved_buf(d.save_index);
          use(s.dst, d.num_inputs);
          break;
        }
        case PONNI_B200_BINOP_ADD: {
          StepDesc& s = new_step(STEP_ADD);
          s.nin = s.nout = d.num_inputs;
          s.src = cur;
          s.aux = saved_buf(d.save_index);
          break;
        }
        case PONNI_B200_BINOP_CONCATENATE: {
          StepDesc& s = new_step(STEP_CONCAT);
          s.nin = d.num_inputs;
          s.nout = d.num_outputs;
          s.flags = (d.flags & PONNI_B200_FLAG_AFTER) ? CONCAT_AFTER : 0;
          s.src = cur;
          s.aux = saved_buf(d.save_index);
          s.dst = other(cur);
          use(s.dst, d.num_outputs);
          cur = s.dst;
          break;
        }
        case PONNI_B200_BINOP_PROJECTION_ADD: {
          // out[i] = in[i] + (bias[i] + sum_k W[k][i] * saved[k]), in place on
          // the main state: each element is read and written by one thread.
          StepDesc& s = new_step(STEP_DENSE);
          s.nin = d.aux;
          s.nout = d.num_inputs;
          s.nout_pad = (int)align_up(d.num_inputs, kTO);
          s.src = saved_buf(d.save_index);
          s.dst = cur;
          s.aux = cur;
          s.flags = DENSE_INIT_BIAS | DENSE_ADD_RESIDUAL | DENSE_FAST_EPI;
          s.fast_act = EPI_NONE;
          s.w_off = append_matrix(Ly.params.data(), d.aux, d.num_inputs, s.nout_pad);
          s.b_off = append(Ly.params.data() + (size_t)d.aux * d.num_inputs * esz, d.num_inputs);
          s.epi_first = p.n_epi;
          s.n_epi = 0;
          break;
        }
        default: return fail(std::string("unsupported layer ") + layer_label(d.kind));
      }
      ++i;
    }
    if (!last_to_global) p.final_buf = cur;
    p.n_buffers = BUF_SAVED0 + n_saved_buf;
    if (p.n_buffers > kMaxBuffers) return fail("too many saved states");
    return PONNI_B200_OK;
  }
};

}  // namespace

// Select the model's device and create its stream on first use, so that a
// model can be built, validated and (de)serialised on a machine without GPU.
ponni_b200_status pb_ensure_cuda(ponni_b200_model* m) {
  cudaError_t e = cudaSetDevice(m->device);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail(m, e, "cudaSetDevice");
  }
  if (!m->own_stream) {
    e = cudaStreamCreateWithFlags(&m->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_fail(m, e, "cudaStreamCreate");
    if (!m->stream) m->stream = m->own_stream;
  }
  return PONNI_B200_OK;
}

ponni_b200_status pb_check_device_error(ponni_b200_model* m) {
  if (!m->err_dev) return PONNI_B200_OK;
  int flag = 0;
  // Plain synchronous copies of one word (no allocation).
  cudaError_t e = cudaMemcpy(&flag, m->err_dev, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(m, e, "error word read");
  if (!flag) return PONNI_B200_OK;
  cudaMemset(m->err_dev, 0, sizeof(int));
  return pb_fail(m, PONNI_B200_ERR_DEVICE,
                 "a tensor-core kernel's bounded wait gave up (device error code " + std::to_string(flag) +
                     "); results are invalid");
}

// Build (or rebuild after a parameter change) the Program, pick the batch
// tile and where the parameters live, upload the packed parameters.
ponni_b200_status pb_plan(ponni_b200_model* m) {
  if (m->planned && !m->params_dirty) return PONNI_B200_OK;
  ponni_b200_status st = pb_validate(m);
  if (st) return st;
  st = pb_ensure_cuda(m);
  if (st) return st;
  // Parameters updated from device memory: read them back before re-packing.
  st = pb_pull_params(m);
  if (st) return st;
  const size_t esz = dtype_bytes(m->dtype);
  std::vector<unsigned char> packed;
  m->pmap.clear();
  m->pmap.esz = esz;
  m->pmap_uploaded = false;
  {
    int64_t base = 0;
    for (const auto& L : m->layers) {
      const int64_t n = L.num_trainable();
      if (n == 0) continue;
      m->pmap.ranges.push_back({L.params.data(), L.params.data() + (size_t)n * esz, base});
      base += n;
    }
  }
  Planner pl{m, m->prog, packed, esz};
  pl.rec = &m->pmap;
  st = pl.run();
  if (st) return st;
  Program& p = m->prog;
  packed.resize(align_up((int64_t)packed.size() + 16, 16), 0);  // >= 16 bytes, multiple of 16
  const size_t param_bytes = packed.size();
  p.n_params = (int32_t)(param_bytes / esz);

  // Candidates: batch tile 128 / 64 / 32, parameters in shared or global
  // memory.  Preferred: at least two resident CTAs (16 warps per SM to hide
  // shared-memory and FMA latency), then the largest tile (a 256-thread CTA
  // needs 128 columns to keep every thread busy on 64-wide layers), then the
  // higher occupancy, then the parameters on chip.  Measured: cfg2 (fp32
  // 30-64-64-64-10) 128 columns with parameters in L1/L2 at 2 CTAs/SM beat
  // the same tile with parameters in shared memory at 1 CTA/SM by 1.24x; cfg4
  // (128-wide residual blocks) 64 columns at 2 CTAs/SM beat 128 columns at 1
  // CTA/SM by 1.69x.
  // PONNI_B200_TILE="bt,params_in_smem" overrides (tuning aid).
  int force_bt = 0, force_psm = -1;
  if (const char* env = getenv("PONNI_B200_TILE")) sscanf(env, "%d,%d", &force_bt, &force_psm);
  int best_bt = 0, best_occ = 0, best_psm = 0;
  size_t best_smem = 0;
  auto better = [&](int bt, int occ, int psm) {
    if (best_bt == 0) return true;
    const int a = std::min(occ, 2), b = std::min(best_occ, 2);
    if (a != b) return a > b;
    if (bt != best_bt) return bt > best_bt;
    if (occ != best_occ) return occ > best_occ;
    return psm > best_psm;
  };
  for (int bt : {128, 64, 32}) {
    if (force_bt && bt != force_bt) continue;
    for (int psm : {1, 0}) {
      if (force_psm >= 0 && psm != force_psm) continue;
      size_t smem = 0;
      for (int b = 0; b < p.n_buffers; ++b) smem += (size_t)align_up((int64_t)pl.width[b] * bt * esz, 128);
      if (psm) smem += param_bytes;
      if (smem > 227 * 1024) continue;
      int occ = tile_forward_occupancy((int)m->dtype, smem);
      if (occ <= 0 || !better(bt, occ, psm)) continue;
      best_bt = bt;
      best_occ = occ;
      best_psm = psm;
      best_smem = smem;
    }
  }
  if (best_bt == 0)
    return pb_fail(m, PONNI_B200_ERR_UNSUPPORTED,
                   "layer widths exceed the on-chip tile capacity (shared memory) of the fused kernel");
  p.bt = best_bt;
  size_t off = 0;
  for (int b = 0; b < kMaxBuffers; ++b) {
    p.buf_width[b] = b < p.n_buffers ? pl.width[b] : 0;
    p.buf_off[b] = (int)(off / esz);
    if (b < p.n_buffers) off += (size_t)align_up((int64_t)pl.width[b] * best_bt * esz, 128);
  }
  p.params_in_smem = best_psm;
  p.param_smem_off = (int)(off / esz);
  m->smem_bytes = best_smem;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device);
  m->num_sms = sms;
  m->grid = sms * best_occ;
  if (packed.size() > m->packed_dev_bytes) {
    if (m->packed_dev) {
      cudaStreamSynchronize(m->stream);
      cudaFree(m->packed_dev);
    }
    m->packed_dev = nullptr;
    m->packed_dev_bytes = 0;
    cudaError_t e = cudaMalloc(&m->packed_dev, packed.size());
    if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(parameters)");
    m->packed_dev_bytes = packed.size();
  }
  // Stream-ordered after any forward still reading the old parameters.
  cudaError_t e = cudaMemcpyAsync(m->packed_dev, packed.data(), packed.size(), cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return cuda_fail(m, e, "parameter upload");
  m->packed_host.swap(packed);

  // Tensor-core dense-chain kernel, when allowed and eligible.
  m->kernel = 1;
  m->tc_why.clear();
  // AUTO: tensor cores for fp32 models (fp32-accurate split arithmetic);
  // fp16/bf16 models keep the reference's per-operation rounding unless the
  // caller asks for fp32 accumulation (ARITH_TENSOR).
  // Narrow chains (every layer at most 16 wide) are bandwidth-bound and stay
  // on the tile kernel under AUTO.
  int widest = 0;
  for (const auto& L : m->layers) widest = std::max(widest, std::max(L.d.num_inputs, L.d.num_outputs));
  const bool want_tc = m->arithmetic == PONNI_B200_ARITH_TENSOR ||
                       (m->arithmetic == PONNI_B200_ARITH_AUTO && m->dtype == PONNI_B200_F32 && widest > 16);
  if (want_tc) {
    std::vector<unsigned char> image;
    // PONNI_B200_TC_STREAM=1 (a test aid) sends eligible 16-bit chains to the
    // streamed-weights kernel even when their weights fit shared memory.
    const char* force_stream = getenv("PONNI_B200_TC_STREAM");
    const bool stream_first = force_stream && force_stream[0] == '1' && m->dtype != PONNI_B200_F32;
    std::string why_tr;
    ParamMap tc_rec;
    tc_rec.ranges = m->pmap.ranges;
    tc_rec.esz = esz;
    if (!stream_first && tc_plan(m, m->tcp, image, m->tc_why, &tc_rec)) {
      if (image.size() > m->tc_image_bytes) {
        if (m->tc_image_dev) cudaFree(m->tc_image_dev);
        m->tc_image_dev = nullptr;
        m->tc_image_bytes = 0;
        e = cudaMalloc(&m->tc_image_dev, image.size());
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(tensor-core parameters)");
        m->tc_image_bytes = image.size();
      }
      if (!m->err_dev) {
        // error word + 7 diagnostic counters (filled only by a build with
        // phase profiling enabled)
        e = cudaMalloc(&m->err_dev, 64);
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(error word)");
        e = cudaMemsetAsync(m->err_dev, 0, 64, m->stream);
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMemset(error word)");
      }
      e = cudaMemcpyAsync(m->tc_image_dev, image.data(), image.size(), cudaMemcpyHostToDevice, m->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
      if (e != cudaSuccess) return cuda_fail(m, e, "tensor-core parameter upload");
      m->tc_grid = m->num_sms;  // one persistent CTA (up to eight tile slots) per SM
      m->kernel = 2;
      // The model-specialised build of the same kernel (NVRTC), when it compiles.
      m->tc_jit = nullptr;
      m->tc_jit_why.clear();
      if (!tc_jit_build(m->tcp, &m->tc_jit, &m->tc_jit_why)) m->tc_jit = nullptr;
      m->pmap.recs.insert(m->pmap.recs.end(), tc_rec.recs.begin(), tc_rec.recs.end());
      m->pmap.overflow |= tc_rec.overflow;
    } else if (m->dtype == PONNI_B200_F32 && !(getenv("PONNI_B200_TC_RESID") && getenv("PONNI_B200_TC_RESID")[0] == '0') &&
               (tc_rec.recs.clear(), tr_plan(m, m->trp, image, why_tr, &tc_rec))) {
      // LayerNorm / residual chains (and fp32 chains too wide for the
      // resident kernel): weights streamed, barriers in the epilogue.
      if (image.size() > m->ts_image_bytes) {
        if (m->ts_image_dev) cudaFree(m->ts_image_dev);
        m->ts_image_dev = nullptr;
        m->ts_image_bytes = 0;
        e = cudaMalloc(&m->ts_image_dev, image.size());
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(streamed tensor-core parameters)");
        m->ts_image_bytes = image.size();
      }
      const size_t scratch = (size_t)m->num_sms * m->trp.scratch_per_cta;
      if (scratch > m->scratch_bytes) {
        if (m->scratch_dev) cudaFree(m->scratch_dev);
        m->scratch_dev = nullptr;
        m->scratch_bytes = 0;
        e = cudaMalloc(&m->scratch_dev, scratch);
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(saved-state scratch)");
        m->scratch_bytes = scratch;
      }
      if (!m->err_dev) {
        e = cudaMalloc(&m->err_dev, 64);
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(error word)");
        e = cudaMemsetAsync(m->err_dev, 0, 64, m->stream);
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMemset(error word)");
      }
      e = cudaMemcpyAsync(m->ts_image_dev, image.data(), image.size(), cudaMemcpyHostToDevice, m->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
      if (e != cudaSuccess) return cuda_fail(m, e, "residual tensor-core parameter upload");
      m->tc_grid = m->num_sms;
      // PONNI_B200_TC_GRID=n caps the persistent grid (a test aid: several
      // tiles per CTA, both tile slots busy, on a small batch).
      if (const char* g = getenv("PONNI_B200_TC_GRID")) m->tc_grid = std::max(1, std::min(m->num_sms, atoi(g)));
      m->kernel = 6;
      m->pmap.recs.insert(m->pmap.recs.end(), tc_rec.recs.begin(), tc_rec.recs.end());
      m->pmap.overflow |= tc_rec.overflow;
    } else if (m->arithmetic == PONNI_B200_ARITH_TENSOR) {
      // Weights beyond shared memory: stream them per layer (16-bit models).
      std::string why2;
      tc_rec.recs.clear();
      if (!ts_plan(m, m->tsp, image, why2, &tc_rec))
        return pb_fail(m, PONNI_B200_ERR_UNSUPPORTED,
                       "tensor-core kernel unavailable: " + (m->tc_why.empty() ? why2 : m->tc_why + "; " + why2));
      if (image.size() > m->ts_image_bytes) {
        if (m->ts_image_dev) cudaFree(m->ts_image_dev);
        m->ts_image_dev = nullptr;
        m->ts_image_bytes = 0;
        e = cudaMalloc(&m->ts_image_dev, image.size());
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(streamed tensor-core parameters)");
        m->ts_image_bytes = image.size();
      }
      if (!m->err_dev) {
        e = cudaMalloc(&m->err_dev, 64);
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(error word)");
        e = cudaMemsetAsync(m->err_dev, 0, 64, m->stream);
        if (e != cudaSuccess) return cuda_fail(m, e, "cudaMemset(error word)");
      }
      e = cudaMemcpyAsync(m->ts_image_dev, image.data(), image.size(), cudaMemcpyHostToDevice, m->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
      if (e != cudaSuccess) return cuda_fail(m, e, "streamed tensor-core parameter upload");
      m->tc_grid = m->num_sms;
      m->kernel = 5;
      m->tc_jit = nullptr;
      m->tc_jit_why.clear();
      if (!ts_jit_build(m->tsp, &m->tc_jit, &m->tc_jit_why)) m->tc_jit = nullptr;
      m->pmap.recs.insert(m->pmap.recs.end(), tc_rec.recs.begin(), tc_rec.recs.end());
      m->pmap.overflow |= tc_rec.overflow;
    }
  }
  // Narrow chains (every width <= 32) stream through registers, unless the
  // tile kernel is forced (PONNI_B200_FORCE_TILE=1, a test aid).
  const char* force_tile = getenv("PONNI_B200_FORCE_TILE");
  if (m->kernel == 1 && !(force_tile && force_tile[0] == '1') && narrow_eligible((int)m->dtype, p, &m->narrow_maxw)) {
    if (!m->prog_dev) {
      e = cudaMalloc(&m->prog_dev, sizeof(Program));
      if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(program)");
    }
    e = cudaMemcpyAsync(m->prog_dev, &p, sizeof(Program), cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e == cudaSuccess) e = narrow_prepare((int)m->dtype, p, m->narrow_maxw, m->num_sms, &m->narrow);
    if (e != cudaSuccess) return cuda_fail(m, e, "narrow kernel preparation");
    m->kernel = 3;
    // Model-specialised form, unless disabled (PONNI_B200_NARROW_JIT=0) or
    // unavailable (then the generic narrow kernel runs).
    const char* jit = getenv("PONNI_B200_NARROW_JIT");
    m->jit_why.clear();
    if (jit && jit[0] == '0') m->jit_why = "disabled by PONNI_B200_NARROW_JIT=0";
    else if (narrow_jit_build((int)m->dtype, p, m->narrow_maxw, m->packed_host, m->num_sms, &m->jit, &m->jit_why))
      m->kernel = 4;
  }
  m->planned = true;
  m->params_dirty = false;
  return PONNI_B200_OK;
}

// Reference get_planned_temporary_size (src/ponni_Inference.h:92-122).
static int planned_temporary_size(const ponni_b200_model* m, int requested) {
  const int L = (int)m->layers.size();
  int mx = 0;
  bool in_tmp1 = false;
  int i = 0;
  while (i < L) {
    const auto& d = m->layers[i].d;
    if (is_dense(d.kind)) {
      int end = i + 1;
      while (end < L && is_pointwise(m->layers[end].d.kind)) ++end;
      if (end == L) return mx;
      bool out_tmp1 = i == 0 ? true : !in_tmp1;
      if (requested == (out_tmp1 ? 0 : 1)) mx = std::max(mx, d.num_outputs);
      i = end;
      in_tmp1 = out_tmp1;
    } else if (i == L - 1) {
      return mx;
    } else {
      bool out_tmp1 = i == 0 ? true : (overwrites_input(d.kind) ? in_tmp1 : !in_tmp1);
      if (requested == (out_tmp1 ? 0 : 1)) mx = std::max(mx, d.num_outputs);
      ++i;
      in_tmp1 = out_tmp1;
    }
  }
  return mx;
}

// ---------------------------------------------------------------------------
// Reference weight_schema_fingerprint (src/ponni_Inference.h:270-288).
std::string pb_schema_fingerprint(const ponni_b200_model* m) {
  std::ostringstream s;
  s << "ponni-template-model-v1\n";
  for (size_t i = 0; i < m->layers.size(); ++i) {
    const auto& L = m->layers[i];
    s << i << '\t' << layer_label(L.d.kind) << '\t' << L.d.num_inputs << '\t' << L.d.num_outputs << '\t'
      << L.num_trainable() << '\n';
  }
  const std::string text = s.str();
  uint64_t h = UINT64_C(14695981039346656037);
  for (unsigned char c : text) {
    h ^= c;
    h *= UINT64_C(1099511628211);
  }
  char buf[32];
  snprintf(buf, sizeof buf, "fnv1a64:%016llx", (unsigned long long)h);
  return buf;
}

extern "C" {

int ponni_b200_abi_version(void) { return PONNI_B200_ABI_VERSION; }

ponni_b200_status ponni_b200_device_count(int* count) {
  if (!count) return PONNI_B200_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    cudaGetLastError();
    return PONNI_B200_ERR_CUDA;
  }
  return PONNI_B200_OK;
}

const char* ponni_b200_create_error(void) { return g_create_error.c_str(); }

ponni_b200_status ponni_b200_model_create(const ponni_b200_layer_desc* layers, int num_layers,
                                          ponni_b200_dtype dtype, int device, ponni_b200_model** out_model) {
  g_create_error.clear();
  if (!out_model) {
    g_create_error = "out_model is NULL";
    return PONNI_B200_ERR_INVALID_ARGUMENT;
  }
  *out_model = nullptr;
  if (!layers || num_layers <= 0) {
    g_create_error = "a model needs at least one layer";
    return PONNI_B200_ERR_INVALID_ARGUMENT;
  }
  if (dtype_bytes(dtype) == 0) {
    g_create_error = "unknown dtype";
    return PONNI_B200_ERR_INVALID_ARGUMENT;
  }
  auto* m = new ponni_b200_model();
  m->dtype = dtype;
  m->device = device;
  const size_t esz = dtype_bytes(dtype);
  for (int i = 0; i < num_layers; ++i) {
    Layer L;
    L.d = layers[i];
    L.d.params = nullptr;
    for (int k = 0; k < 3; ++k) {
      L.d.scalar[k] = round_to_dtype(dtype, layers[i].scalar[k]);
      L.raw_scalar[k] = layers[i].scalar[k];
    }
    int64_t n = L.num_params();
    if (n < 0 || (n > 0 && (L.d.num_inputs <= 0 || L.d.num_outputs <= 0 ||
                            (L.d.kind == PONNI_B200_BINOP_PROJECTION_ADD && L.d.aux <= 0))))
      n = 0;
    if (n > 0) {
      if (!layers[i].params) {
        g_create_error = std::string("layer ") + std::to_string(i) + " (" + layer_label(L.d.kind) +
                         ") needs a parameter pointer";
        delete m;
        return PONNI_B200_ERR_INVALID_ARGUMENT;
      }
      L.params.resize((size_t)n * esz);
      memcpy(L.params.data(), layers[i].params, L.params.size());
    }
    m->layers.push_back(std::move(L));
  }
  *out_model = m;
  return PONNI_B200_OK;
}

void ponni_b200_model_destroy(ponni_b200_model* m) {
  if (!m) return;
  DeviceGuard guard(m->device);
  if (m->own_stream || m->packed_dev || m->stage_dev || m->tc_image_dev || m->err_dev || m->prog_dev ||
      m->ts_image_dev || m->scratch_dev || m->pmap_dev.recs || m->pmap_dev.staging) {
    DeviceGuard guard(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->copy_stream) cudaStreamSynchronize(m->copy_stream);
    if (m->packed_dev) cudaFree(m->packed_dev);
    if (m->prog_dev) cudaFree(m->prog_dev);
    if (m->ts_image_dev) cudaFree(m->ts_image_dev);
    if (m->scratch_dev) cudaFree(m->scratch_dev);
    if (m->stage_dev) cudaFree(m->stage_dev);
    if (m->tc_image_dev) cudaFree(m->tc_image_dev);
    if (m->err_dev) cudaFree(m->err_dev);
    pb_free_param_map(m);
    if (m->copy_stream) cudaStreamDestroy(m->copy_stream);
    if (m->own_stream) cudaStreamDestroy(m->own_stream);
  }
  delete m;
}

const char* ponni_b200_last_error(const ponni_b200_model* m) { return m ? m->last_error.c_str() : ""; }

ponni_b200_status ponni_b200_model_validate(ponni_b200_model* m) {
  if (!m) return PONNI_B200_ERR_INVALID_ARGUMENT;
  return pb_validate(m);
}

int ponni_b200_num_inputs(const ponni_b200_model* m) { return m ? m->layers.front().d.num_inputs : 0; }
int ponni_b200_num_outputs(const ponni_b200_model* m) { return m ? m->layers.back().d.num_outputs : 0; }
int ponni_b200_num_layers(const ponni_b200_model* m) { return m ? (int)m->layers.size() : 0; }
ponni_b200_dtype ponni_b200_model_dtype(const ponni_b200_model* m) { return m ? m->dtype : PONNI_B200_F32; }

void* ponni_b200_model_stream(const ponni_b200_model* m) {
  if (!m) return nullptr;
  if (!m->stream) {
    DeviceGuard guard(m->device);
    pb_ensure_cuda(const_cast<ponni_b200_model*>(m));
  }
  return (void*)m->stream;
}

ponni_b200_status ponni_b200_model_set_stream(ponni_b200_model* m, void* stream) {
  if (!m) return PONNI_B200_ERR_INVALID_ARGUMENT;
  if (!stream) {
    DeviceGuard guard(m->device);
    ponni_b200_status st = pb_ensure_cuda(m);
    if (st) return st;
  }
  m->stream = stream ? (cudaStream_t)stream : m->own_stream;
  return PONNI_B200_OK;
}

ponni_b200_status ponni_b200_model_synchronize(ponni_b200_model* m) {
  if (!m) return PONNI_B200_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(m->device);
  ponni_b200_status st = pb_ensure_cuda(m);
  if (st) return st;
  cudaError_t e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return cuda_fail(m, e, "cudaStreamSynchronize");
  return pb_check_device_error(m);
}

ponni_b200_status ponni_b200_forward(ponni_b200_model* m, const void* input, int64_t in_ld, void* output,
                                     int64_t out_ld, int64_t batch, void* stream) {
  if (!m) return PONNI_B200_ERR_INVALID_ARGUMENT;
  if (batch <= 0) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "Inference requires a nonzero batch size");
  if (batch > INT32_MAX) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "batch size exceeds INT_MAX");
  if (!input || !output) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "input/output pointer is NULL");
  if (in_ld < batch || out_ld < batch)
    return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "row stride smaller than the batch size");
  // Launch on the model's device; the caller's current device is restored.
  DeviceGuard guard(m->device);
  ponni_b200_status st = pb_plan(m);
  if (st) return st;
  // Reference ensure_internal_state_capacity (src/ponni_Inference.h:197-199).
  if (batch > m->capacity) m->capacity = batch;
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  cudaError_t e;
  if (m->kernel == 2) {
    const int64_t ntiles = (batch + kTcM - 1) / kTcM;
    const int grid = (int)std::min<int64_t>(m->tc_grid, (ntiles + m->tcp.slots - 1) / m->tcp.slots);
    e = m->tc_jit ? launch_tc_forward_jit(m->tc_jit, m->tcp, m->tc_image_dev, input, in_ld, output, out_ld, batch,
                                          grid, m->err_dev, s)
                  : launch_tc_forward(m->tcp, m->tc_image_dev, input, in_ld, output, out_ld, batch, grid, m->err_dev, s);
  } else if (m->kernel == 5) {
    const int64_t ntiles = (batch + kTcM - 1) / kTcM;
    const int grid = (int)std::min<int64_t>(m->tc_grid, ntiles);
    e = m->tc_jit ? launch_ts_forward_jit(m->tc_jit, m->tsp, m->ts_image_dev, input, in_ld, output, out_ld, batch,
                                          grid, m->err_dev, s)
                  : launch_ts_forward(m->tsp, m->ts_image_dev, input, in_ld, output, out_ld, batch, grid, m->err_dev, s);
  } else if (m->kernel == 6) {
    const int64_t ntiles = (batch + kTcM - 1) / kTcM;
    const int grid = (int)std::min<int64_t>(m->tc_grid, ntiles);
    e = launch_tr_forward(m->trp, m->ts_image_dev, m->scratch_dev, input, in_ld, output, out_ld, batch, grid,
                          m->err_dev, s);
  } else if (m->kernel == 4) {
    e = narrow_jit_launch(m->jit, input, in_ld, output, out_ld, batch, s);
  } else if (m->kernel == 3) {
    e = launch_narrow_forward(m->narrow, static_cast<const Program*>(m->prog_dev), m->packed_dev, input, in_ld,
                              output, out_ld, batch, s);
  } else {
    const int64_t ntiles = (batch + m->prog.bt - 1) / m->prog.bt;
    const int grid = (int)std::min<int64_t>(m->grid, ntiles);
    e = launch_tile_forward((int)m->dtype, m->prog, m->packed_dev, input, in_ld, output, out_ld, batch, grid,
                            m->smem_bytes, s);
  }
  if (e != cudaSuccess) return cuda_fail(m, e, "kernel launch");
  return PONNI_B200_OK;
}

ponni_b200_status ponni_b200_reallocate_internal_state(ponni_b200_model* m, int64_t batch) {
  if (!m) return PONNI_B200_ERR_INVALID_ARGUMENT;
  if (batch < 0)
    return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "Inference internal-state batch size must be nonnegative");
  if (m->stream) {  // reference fences its execution space first
    DeviceGuard guard(m->device);
    cudaStreamSynchronize(m->stream);
  }
  m->capacity = batch;
  return PONNI_B200_OK;
}

int64_t ponni_b200_internal_state_capacity(const ponni_b200_model* m) { return m ? m->capacity : 0; }

int ponni_b200_planned_temporary_size(const ponni_b200_model* m, int which) {
  return m ? planned_temporary_size(m, which) : 0;
}

int ponni_b200_num_saved_states(const ponni_b200_model* m) {
  int n = 0;
  if (m)
    for (const auto& L : m->layers)
      if (is_save(L.d.kind)) n = std::max(n, L.d.save_index + 1);
  return n;
}

int ponni_b200_saved_state_size(const ponni_b200_model* m, int index) {
  int n = 0;
  if (m)
    for (const auto& L : m->layers)
      if (is_save(L.d.kind) && L.d.save_index == index) n = std::max(n, L.d.num_outputs);
  return n;
}

ponni_b200_status ponni_b200_model_set_arithmetic(ponni_b200_model* m, int arithmetic) {
  if (!m || arithmetic < PONNI_B200_ARITH_AUTO || arithmetic > PONNI_B200_ARITH_GENERATED)
    return PONNI_B200_ERR_INVALID_ARGUMENT;
  if (m->arithmetic != arithmetic) {
    m->arithmetic = arithmetic;
    m->params_dirty = true;  // re-plan on the next forward
  }
  return PONNI_B200_OK;
}

ponni_b200_status ponni_b200_model_device_program(ponni_b200_model* m, const void** program, const void** params,
                                                  int* max_width, int* num_buffers) {
  if (!m || !program || !params) return PONNI_B200_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(m->device);
  ponni_b200_status st = pb_plan(m);
  if (st) return st;
  cudaError_t e = cudaSuccess;
  if (!m->prog_dev) {
    e = cudaMalloc(&m->prog_dev, sizeof(Program));
    if (e != cudaSuccess) return cuda_fail(m, e, "cudaMalloc(program)");
  }
  e = cudaMemcpyAsync(m->prog_dev, &m->prog, sizeof(Program), cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  if (e != cudaSuccess) return cuda_fail(m, e, "program upload");
  int w = std::max(m->prog.nin, m->prog.nout);
  for (int b = 0; b < m->prog.n_buffers; ++b) w = std::max(w, m->prog.buf_width[b]);
  *program = m->prog_dev;
  *params = m->packed_dev;
  if (max_width) *max_width = w;
  if (num_buffers) *num_buffers = m->prog.n_buffers;
  return PONNI_B200_OK;
}

int ponni_b200_model_kernel(ponni_b200_model* m) {
  if (!m) return 0;
  DeviceGuard guard(m->device);
  return pb_plan(m) == PONNI_B200_OK ? m->kernel : 0;
}

int ponni_b200_model_specialised(ponni_b200_model* m, const char** why) {
  if (why) *why = "";
  if (!m) return 0;
  DeviceGuard guard(m->device);
  if (pb_plan(m) != PONNI_B200_OK) return 0;
  if (m->kernel == 4) return 1;
  if ((m->kernel == 2 || m->kernel == 5) && m->tc_jit) return 1;
  if (why)
    *why = (m->kernel == 2 || m->kernel == 5) ? m->tc_jit_why.c_str() : m->kernel == 3 ? m->jit_why.c_str() : "";
  return 0;
}

ponni_b200_status ponni_b200_model_diagnostics(ponni_b200_model* m, uint64_t* out, int n) {
  if (!m || !out || n < 0) return PONNI_B200_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < n; ++i) out[i] = 0;
  if (!m->err_dev) return PONNI_B200_OK;
  uint64_t buf[8];
  DeviceGuard guard(m->device);
  cudaError_t e = cudaStreamSynchronize(m->stream);
  if (e == cudaSuccess) e = cudaMemcpy(buf, m->err_dev, 64, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(m, e, "diagnostics read");
  for (int i = 0; i < n && i < 7; ++i) out[i] = buf[1 + i];
  return PONNI_B200_OK;
}

int64_t ponni_b200_scratch_bytes(const ponni_b200_model* m) { return m ? (int64_t)m->scratch_bytes : 0; }

// Tuple-order flattening of set/get_trainable_parameters
// (src/ponni_Inference.h:689-716): each trainable layer consumes the prefix of
// its own size; Matvec is W[in][out] row-major, LayerNorm gamma then beta,
// Binop_Projection_Add W[nsave][nin] then bias.
int64_t ponni_b200_num_trainable_parameters(const ponni_b200_model* m) {
  int64_t n = 0;
  if (m)
    for (const auto& L : m->layers) n += L.num_trainable();
  return n;
}

ponni_b200_status ponni_b200_set_trainable_parameters(ponni_b200_model* m, const void* host, int64_t count) {
  if (!m || (!host && count > 0)) return PONNI_B200_ERR_INVALID_ARGUMENT;
  const int64_t need = ponni_b200_num_trainable_parameters(m);
  if (count < need) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "ERROR: trainable input too small");
  const size_t esz = dtype_bytes(m->dtype);
  const unsigned char* src = static_cast<const unsigned char*>(host);
  for (auto& L : m->layers) {
    const int64_t n = L.num_trainable();
    if (n == 0) continue;
    memcpy(L.params.data(), src, (size_t)n * esz);
    src += (size_t)n * esz;
  }
  m->host_params_stale = false;  // every trainable value was just written
  // A planned model takes the values into its device images directly
  // (pinned staging + device scatter); otherwise the next forward re-plans.
  if (pb_update_params_from_host(m, host, need) == PONNI_B200_OK) return PONNI_B200_OK;
  m->params_dirty = true;
  return PONNI_B200_OK;
}

ponni_b200_status ponni_b200_get_trainable_parameters(ponni_b200_model* m, void* host, int64_t count) {
  if (!m || (!host && count > 0)) return PONNI_B200_ERR_INVALID_ARGUMENT;
  const int64_t need = ponni_b200_num_trainable_parameters(m);
  if (count < need) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "output buffer too small");
  ponni_b200_status st = pb_pull_params(m);  // after updates from device memory
  if (st) return st;
  const size_t esz = dtype_bytes(m->dtype);
  unsigned char* dst = static_cast<unsigned char*>(host);
  for (auto& L : m->layers) {
    const int64_t n = L.num_trainable();
    if (n == 0) continue;
    memcpy(dst, L.params.data(), (size_t)n * esz);
    dst += (size_t)n * esz;
  }
  return PONNI_B200_OK;
}

ponni_b200_status ponni_b200_weight_schema_fingerprint(const ponni_b200_model* m, char* buf, size_t len) {
  if (!m || !buf) return PONNI_B200_ERR_INVALID_ARGUMENT;
  const std::string f = pb_schema_fingerprint(m);
  if (len < f.size() + 1) return PONNI_B200_ERR_INVALID_ARGUMENT;
  memcpy(buf, f.c_str(), f.size() + 1);
  return PONNI_B200_OK;
}

// Reference Inference::print (src/ponni_Inference.h:671-683).
ponni_b200_status ponni_b200_model_summary(const ponni_b200_model* m, char* buf, size_t len) {
  if (!m || !buf || len == 0) return PONNI_B200_ERR_INVALID_ARGUMENT;
  std::ostringstream s;
  s << "Inference model has " << m->layers.size() << " layers -- with " << ponni_b200_num_trainable_parameters(m)
    << " total trainable parameters.\n";
  for (size_t i = 0; i < m->layers.size(); ++i) {
    const auto& L = m->layers[i];
    char line[256];
    snprintf(line, sizeof line, "  %3d: %-15s with %d inputs, %d outputs, and %lld trainable parameters\n",
             (int)i + 1, layer_label(L.d.kind), L.d.num_inputs, L.d.num_outputs, (long long)L.num_trainable());
    s << line;
  }
  const std::string t = s.str();
  const size_t n = std::min(len - 1, t.size());
  memcpy(buf, t.data(), n);
  buf[n] = 0;
  return t.size() < len ? PONNI_B200_OK : PONNI_B200_ERR_INVALID_ARGUMENT;
}

}  // extern "C"
