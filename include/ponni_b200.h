/*
 * libponni_b200 -- C ABI of the B200-native PONNI batched-inference path.
 *
 * A model is a flat list of layer descriptors (the lowered form of PONNI's
 * compile-time layer tuple).  All data is feature-major [features, batch]
 * with the batch index contiguous, exactly as PONNI's LayoutRight Views.
 * Every entry point returns a ponni_b200_status; the text of the last error
 * on a model is available from ponni_b200_last_error().
 *
 * Plain pointers and sizes only: no CUDA, Kokkos or torch types appear in the
 * signatures.  Streams are passed as opaque `void*` (a cudaStream_t; NULL
 * means the model's own stream, so the legacy default stream is passed as
 * cudaStreamLegacy, (void*)0x1).
 *
 * Reference interfaces replaced (paths inside mrnorman/ponni):
 *   ponni_b200_model_create        <- ponni::create_inference_model[_single|_double|_half|_bhalf_precision]
 *                                     src/ponni_create_model.h:21-98, Inference ctor src/ponni_Inference.h:159
 *   ponni_b200_model_validate      <- Inference::validate            src/ponni_Inference.h:719-737
 *   ponni_b200_forward             <- Inference::forward_batch_parallel(input,output)
 *                                     src/ponni_Inference.h:352-389 (async on the model's stream)
 *   ponni_b200_forward_host        <- forward_batch_parallel(create_device_copy(in)) + create_host_copy(out)
 *                                     src/ponni_Inference.h:339-346, src/utils/ponni_view_ops.h:12-37
 *   ponni_b200_reallocate_internal_state / ponni_b200_internal_state_capacity
 *                                  <- src/ponni_Inference.h:169-180, 197-199
 *   ponni_b200_planned_temporary_size / ponni_b200_saved_state_size
 *                                  <- get_planned_temporary_size / get_saved_state_size
 *                                     src/ponni_Inference.h:93-122, 204-223
 *   ponni_b200_num_trainable_parameters, _set/_get_trainable_parameters
 *                                  <- src/ponni_Inference.h:245-253, 689-716
 *   ponni_b200_weight_schema_fingerprint <- src/ponni_Inference.h:270-288
 *   ponni_b200_model_save_weights / _load_weights
 *                                  <- Inference::save_weights / load_weights src/ponni_Inference.h:295-333
 *                                     (.ponni Safetensors profile, src/utils/ponni_safetensors.h:175-407)
 *   ponni_b200_read_ponni_tensor   <- load_ponni_tensor<N> src/utils/ponni_safetensors.h:409-444
 *   ponni_b200_model_summary       <- Inference::print src/ponni_Inference.h:671-683
 *   ponni_b200_set/_get_trainable_parameters_device, ponni_b200_check_parameters
 *                                  <- generated GeneratedModel::set_parameters / get_parameters /
 *                                     refresh_half_parameters / parameters_are_finite /
 *                                     parameters_synchronized, src/generator/kokkos_nn/emitter.py:1769-1895
 *   ponni_b200_model_set_arithmetic(PONNI_B200_ARITH_GENERATED)
 *                                  <- the generated struct's infer_batch / infer_batch_half2 arithmetic,
 *                                     emitter.py:704-708, 975-983
 *   ponni_b200_model_device_program <- forward_batch_parallel_in_kernel src/ponni_Inference.h:392-408, 592-604
 */
#ifndef PONNI_B200_H
#define PONNI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define PONNI_B200_ABI_VERSION 1

typedef enum {
  PONNI_B200_OK = 0,
  PONNI_B200_ERR_INVALID_ARGUMENT = 1, /* bad pointer / size / layer list */
  PONNI_B200_ERR_VALIDATION = 2,       /* layer dimension mismatch (reference aborts) */
  PONNI_B200_ERR_UNSUPPORTED = 3,      /* layer combination no kernel supports */
  PONNI_B200_ERR_CUDA = 4,             /* CUDA runtime error */
  PONNI_B200_ERR_IO = 5,               /* .ponni file open/read/write/format error */
  PONNI_B200_ERR_MISMATCH = 6,         /* .ponni fingerprint/dtype/shape mismatch */
  PONNI_B200_ERR_DEVICE = 7            /* device-side error flag (bounded wait gave up) */
} ponni_b200_status;

/* Arithmetic type of the model (`real` in ponni::Inference). */
typedef enum {
  PONNI_B200_F32 = 0,  /* create_inference_model / _single_precision */
  PONNI_B200_F64 = 1,  /* _double_precision */
  PONNI_B200_F16 = 2,  /* _half_precision  (Kokkos::Experimental::half_t) */
  PONNI_B200_BF16 = 3  /* _bhalf_precision (Kokkos::Experimental::bhalf_t) */
} ponni_b200_dtype;

/* Layer kinds; labels in the comments are each layer's get_label(). */
typedef enum {
  PONNI_B200_MATVEC = 0,             /* "Matvec"   params W[in][out] row-major       src/layers/ponni_Matvec.h */
  PONNI_B200_BIAS = 1,               /* "Bias"     params b[n]                       src/layers/ponni_Bias.h */
  PONNI_B200_RELU = 2,               /* "ReLU"                                       src/layers/ponni_Relu.h */
  PONNI_B200_LEAKY_RELU = 3,         /* "LeakyReLU" scalar0 = negative_slope         src/layers/ponni_LeakyRelu.h */
  PONNI_B200_ELU = 4,                /* "ELU"      scalar0 = alpha                   src/layers/ponni_Elu.h */
  PONNI_B200_SELU = 5,               /* "SELU"                                       src/layers/ponni_Selu.h */
  PONNI_B200_GELU = 6,               /* "GELU"     flags bit1 = approximate (tanh)   src/layers/ponni_Gelu.h */
  PONNI_B200_SILU = 7,               /* "SiLU"                                       src/layers/ponni_Silu.h */
  PONNI_B200_SIGMOID = 8,            /* "Sigmoid"                                    src/layers/ponni_Sigmoid.h */
  PONNI_B200_TANH = 9,               /* "Tanh"                                       src/layers/ponni_Tanh.h */
  PONNI_B200_SOFTPLUS = 10,          /* "Softplus" scalar0 = beta                    src/layers/ponni_Softplus.h */
  PONNI_B200_HARD_SIGMOID = 11,      /* "HardSigmoid" scalar0 = alpha, scalar1 = beta src/layers/ponni_HardSigmoid.h */
  PONNI_B200_HARD_SWISH = 12,        /* "HardSwish"                                  src/layers/ponni_HardSwish.h */
  PONNI_B200_MISH = 13,              /* "Mish"                                       src/layers/ponni_Mish.h */
  PONNI_B200_LAYER_NORM = 14,        /* "LayerNorm" params gamma[n] then beta[n]; scalar0 = epsilon */
  PONNI_B200_MIN_MAX_NORM = 15,      /* "MinMaxNorm" scalar0 = out_min, scalar1 = out_max, scalar2 = epsilon */
  PONNI_B200_SOFTMAX = 16,           /* "Softmax"                                    src/layers/ponni_Softmax.h */
  PONNI_B200_LOG_SOFTMAX = 17,       /* "LogSoftmax"                                 src/layers/ponni_LogSoftmax.h */
  PONNI_B200_SAVE_STATE = 18,        /* "Save_State" save_index = ISAVE              src/layers/ponni_Save_State.h */
  PONNI_B200_BINOP_ADD = 19,         /* "Binop_Add"  save_index = ISAVE              src/layers/ponni_Binop_Add.h */
  PONNI_B200_BINOP_CONCATENATE = 20, /* "Binop_Concatenate" flags bit2 = after; num_outputs = n1 + n2 */
  PONNI_B200_BINOP_PROJECTION_ADD = 21 /* "Binop_Projection_Add" params W[nsave][nin] then bias[nin];
                                          num_outputs = nin, aux = nsave */
} ponni_b200_layer_kind;

#define PONNI_B200_FLAG_TRAINABLE 0x1   /* parameters take part in the trainable vector */
#define PONNI_B200_FLAG_APPROXIMATE 0x2 /* GELU tanh approximation */
#define PONNI_B200_FLAG_AFTER 0x4       /* Binop_Concatenate: saved state goes after the input */

typedef struct {
  int32_t kind;        /* ponni_b200_layer_kind */
  int32_t num_inputs;  /* layer get_num_inputs() */
  int32_t num_outputs; /* layer get_num_outputs() */
  int32_t save_index;  /* Save_State / Binop_* template ISAVE, else -1 */
  int32_t aux;         /* Binop_Projection_Add: number of saved inputs; else 0 */
  int32_t flags;       /* PONNI_B200_FLAG_* */
  double scalar[3];    /* per-kind scalars (see kinds), rounded to the model dtype */
  const void* params;  /* host pointer, model dtype, canonical flattened order; NULL if none */
} ponni_b200_layer_desc;

typedef struct ponni_b200_model ponni_b200_model;

/* Library / device information. */
int ponni_b200_abi_version(void);
ponni_b200_status ponni_b200_device_count(int* count);

/* Create a model for `device` (CUDA ordinal).  Parameters are copied; the
 * descriptor array and its params may be freed afterwards.  No CUDA call is
 * made until the first forward, so models can be built, validated and
 * (de)serialised on a machine without a GPU. */
ponni_b200_status ponni_b200_model_create(const ponni_b200_layer_desc* layers, int num_layers,
                                          ponni_b200_dtype dtype, int device,
                                          ponni_b200_model** out_model);
void ponni_b200_model_destroy(ponni_b200_model* model);
const char* ponni_b200_last_error(const ponni_b200_model* model);
/* Error text of the last failed ponni_b200_model_create on this thread. */
const char* ponni_b200_create_error(void);

/* Layer-by-layer size checks, reference Inference::validate. */
ponni_b200_status ponni_b200_model_validate(ponni_b200_model* model);

int ponni_b200_num_inputs(const ponni_b200_model* model);
int ponni_b200_num_outputs(const ponni_b200_model* model);
int ponni_b200_num_layers(const ponni_b200_model* model);
ponni_b200_dtype ponni_b200_model_dtype(const ponni_b200_model* model);

/* The model's own CUDA stream (cudaStream_t as void*); `stream` arguments of
 * NULL below mean this stream, matching the reference's stored execution
 * space instance. */
void* ponni_b200_model_stream(const ponni_b200_model* model);
ponni_b200_status ponni_b200_model_set_stream(ponni_b200_model* model, void* stream);
/* Waits for the model's stream; reports PONNI_B200_ERR_DEVICE if a kernel
 * recorded a device-side error (a bounded wait that gave up). */
ponni_b200_status ponni_b200_model_synchronize(ponni_b200_model* model);

/* Arithmetic / kernel selection (no counterpart in the reference, which has
 * one Kokkos kernel):
 *   AUTO      -- fp32 models: tensor cores (tcgen05) for dense chains that
 *                fit the kernel, on an exact three-way bf16 split of every
 *                operand (fp32-level accuracy); fp16/bf16 models: the tile
 *                kernel with the reference's per-operation rounding;
 *   REFERENCE -- always the tile kernel: the reference's arithmetic order
 *                (fp16/bf16 accumulate in the model type, per operation);
 *   TENSOR    -- require the tensor-core kernel (forward fails otherwise);
 *                fp16/bf16 models then accumulate in fp32;
 *   GENERATED -- the arithmetic of the reference's generated (AOT) model
 *                struct (src/generator/kokkos_nn/emitter.py:693-735,
 *                :967-1010): a Matvec followed by a Bias starts its sum at
 *                the bias, and fp16/bf16 models accumulate with one fused
 *                multiply-add per product in the model type (TwoHalf::fma);
 *                the tile kernel. */
typedef enum {
  PONNI_B200_ARITH_AUTO = 0,
  PONNI_B200_ARITH_REFERENCE = 1,
  PONNI_B200_ARITH_TENSOR = 2,
  PONNI_B200_ARITH_GENERATED = 3
} ponni_b200_arithmetic;
ponni_b200_status ponni_b200_model_set_arithmetic(ponni_b200_model* model, int arithmetic);
/* Kernel the next forward uses (plans the model): 1 = tile kernel (SIMT),
 * 2 = tensor-core kernel, 3 = narrow streaming kernel (chains at most 32
 * wide), 4 = the narrow kernel specialised to this model's structure and
 * compiled at plan time with NVRTC (the counterpart of the reference's
 * per-model code generator; PONNI_B200_NARROW_JIT=0 disables it), 5 = the
 * tensor-core kernel with the weights streamed through shared memory layer by
 * layer (16-bit chains whose weights exceed shared memory, ARITH_TENSOR);
 * 0 on a planning error (see last_error). */
int ponni_b200_model_kernel(ponni_b200_model* model);

/* 1 when the kernel the next forward uses was compiled for this model's
 * structure at plan time (NVRTC): kernel 4, or kernels 2 and 5 in their
 * model-specialised builds (layer count, widths, activations as compile-time
 * constants; PONNI_B200_TC_JIT=0 disables them); 0 otherwise, with the reason
 * in `why` (a static-lifetime string owned by the model, may be empty) when
 * `why` is not NULL.  Plans the model.  No reference counterpart: this
 * library's diagnostic. */
int ponni_b200_model_specialised(ponni_b200_model* model, const char** why);

/* Diagnostic counters of the tensor-core kernel (up to 7 values; per-phase
 * cycle sums in a build with -DPONNI_B200_TC_PROFILE, zeros otherwise). */
ponni_b200_status ponni_b200_model_diagnostics(ponni_b200_model* model, uint64_t* out, int n);

/* In-kernel device API (include/ponni_b200_device.cuh): plans the model and
 * returns device pointers to its lowered program and packed parameters (valid
 * until the parameters change or the model is destroyed), the widest state
 * width and the number of state buffers, for evaluating samples inside an
 * application's own kernel.  Replaces Inference::forward_batch_parallel_in_kernel
 * (src/ponni_Inference.h:392-408, :592-604) and the generated model's infer_one. */
ponni_b200_status ponni_b200_model_device_program(ponni_b200_model* model, const void** program, const void** params,
                                                  int* max_width, int* num_buffers);

/* Device-resident forward: input [num_inputs, batch] with row stride in_ld
 * elements, output [num_outputs, batch] with row stride out_ld, both device
 * pointers in the model dtype.  Enqueued on `stream`; returns without a fence
 * (reference forward_batch_parallel semantics).  batch == 0 is an error. */
ponni_b200_status ponni_b200_forward(ponni_b200_model* model, const void* input, int64_t in_ld,
                                     void* output, int64_t out_ld, int64_t batch, void* stream);

/* Host-resident forward: copies host input to the device, runs the model and
 * copies the result back, pipelined in column chunks over two streams.
 * Synchronous: returns when `output` holds the result.  Pinned host memory
 * gives full PCIe bandwidth; pageable memory works too. */
ponni_b200_status ponni_b200_forward_host(ponni_b200_model* model, const void* input, int64_t in_ld,
                                          void* output, int64_t out_ld, int64_t batch);

/* Host-buffer forward that allocates nothing (no counterpart in the
 * reference).  For callers that cannot allocate device memory while they
 * run inference -- an application that gives all of its GPU memory to its
 * own pool at start-up, a solver whose memory budget is fixed before its
 * time loop, or code where a cudaMalloc would synchronise the device at the
 * wrong moment.  Same arguments and result as ponni_b200_forward_host, but
 * the input and output are staged in a static 64 MiB device array that the
 * library holds on every GPU that loads it, until the process exits, and the
 * copies and the kernel run on the model's own stream (no second stream).
 *  - The model must already be prepared: call ponni_b200_model_kernel() once
 *    (it uploads the parameters, which allocates) before the first call, and
 *    again after changing parameters; otherwise this returns an error.
 *  - batch * (num_inputs + num_outputs) * element size must fit in 64 MiB;
 *    larger batches are rejected with an error naming the limit (split them).
 *  - The first call on a device looks up the array's device address; make
 *    that first call before any stream capture.
 *  - Every call, from any model on the same device, shares the array: calls
 *    that overlap on the GPU (other threads, other streams) race.  Each call
 *    overwrites the staged input and output it uses, so nothing needs to be
 *    cleared between calls. */
ponni_b200_status ponni_b200_forward_host_static(ponni_b200_model* model, const void* input, int64_t in_ld,
                                                 void* output, int64_t out_ld, int64_t batch);

/* Scratch capacity, reference semantics: grows on demand to the largest batch
 * seen, shrinks exactly on an explicit call, 0 releases. */
ponni_b200_status ponni_b200_reallocate_internal_state(ponni_b200_model* model, int64_t batch);
int64_t ponni_b200_internal_state_capacity(const ponni_b200_model* model);
/* Planned feature extents of the reference's tmp1 (which=0) / tmp2 (which=1)
 * ping-pong buffers and of saved state `index`; 0 = not needed. */
int ponni_b200_planned_temporary_size(const ponni_b200_model* model, int which);
int ponni_b200_saved_state_size(const ponni_b200_model* model, int index);
int ponni_b200_num_saved_states(const ponni_b200_model* model);
/* Bytes of device scratch currently allocated: 0 unless the program is an
 * fp32 residual chain with two distinct saved states (the residual
 * tensor-core kernel keeps a single saved state on chip). */
int64_t ponni_b200_scratch_bytes(const ponni_b200_model* model);

/* Trainable parameters in tuple (declaration) order, model dtype, host memory. */
int64_t ponni_b200_num_trainable_parameters(const ponni_b200_model* model);
ponni_b200_status ponni_b200_set_trainable_parameters(ponni_b200_model* model, const void* host,
                                                      int64_t count);
ponni_b200_status ponni_b200_get_trainable_parameters(ponni_b200_model* model, void* host,
                                                      int64_t count);

/* Parameter updates of a planned model (one that has run a forward or been
 * prepared by ponni_b200_model_kernel) go straight into its device images:
 * ponni_b200_set_trainable_parameters stages the host values in pinned memory
 * and scatters them on the model stream without a re-plan (replaces the
 * reference's set_trainable_parameters + re-upload, src/ponni_Inference.h:689-703,
 * and the load path of load_weights, :295-316).
 *
 * _device: `src` is device-accessible memory holding `count` >= the
 * trainable count values of `src_dtype` in tuple order; each is converted to
 * the model dtype (fp64 kept, other types through fp32) and written into
 * every device image on `stream` (NULL: the model stream; another stream is
 * joined into the model stream).  Counterpart of the generated model's
 * set_parameters(View, execution space), emitter.py:1826-1866.  The host
 * copy is read back only when needed (get_trainable_parameters, save, a
 * re-plan). */
ponni_b200_status ponni_b200_set_trainable_parameters_device(ponni_b200_model* model, const void* src,
                                                             ponni_b200_dtype src_dtype, int64_t count,
                                                             void* stream);
/* Trainable parameters in tuple order converted to `dst_dtype` into
 * device-accessible `dst`, on `stream` (generated get_parameters,
 * emitter.py:1787-1825). */
ponni_b200_status ponni_b200_get_trainable_parameters_device(ponni_b200_model* model, void* dst,
                                                             ponni_b200_dtype dst_dtype, int64_t count,
                                                             void* stream);
/* Synchronous check of the device images: `mismatches` = image locations
 * (tensor-core weight parts and biases, the specialised narrow kernel's
 * argument block) that differ from the encoding of the packed parameter;
 * `nonfinite` = trainable values that are NaN or infinite.  Counterparts of
 * parameters_synchronized and parameters_are_finite, emitter.py:1868-1895.
 * Either pointer may be NULL. */
ponni_b200_status ponni_b200_check_parameters(ponni_b200_model* model, int64_t* mismatches,
                                              int64_t* nonfinite);

/* "fnv1a64:%016x" of the reference's template schema text; buf >= 25 bytes. */
ponni_b200_status ponni_b200_weight_schema_fingerprint(const ponni_b200_model* model, char* buf,
                                                       size_t len);
ponni_b200_status ponni_b200_model_save_weights(ponni_b200_model* model, const char* path);
ponni_b200_status ponni_b200_model_load_weights(ponni_b200_model* model, const char* path);

/* Read one F32/F64 tensor of any .ponni file as float, after the full
 * structural, schema-fingerprint and checksum checks of the reference's
 * PonniFile::load.  `shape` receives up to 4 extents, `rank` the rank; `out`
 * (capacity elements) may be NULL to query the shape.  `err` receives the
 * reason on failure. */
ponni_b200_status ponni_b200_read_ponni_tensor(const char* path, const char* name, float* out, size_t capacity,
                                               int64_t* shape, int* rank, char* err, size_t err_len);

/* Model summary text, reference Inference::print. */
ponni_b200_status ponni_b200_model_summary(const ponni_b200_model* model, char* buf, size_t len);

/* Synthetic input generator for benchmarks and shards: fills a device
 * [rows, cols] block (row stride ld, model-dtype elements) with a
 * counter-based hash RNG keyed by (seed, row, col0 + col), so any GPU can
 * regenerate any column range.  dist 0 = N(0,1), 1 = U(lo, hi). */
ponni_b200_status ponni_b200_fill_synthetic(ponni_b200_dtype dtype, void* device_ptr, int64_t rows,
                                            int64_t cols, int64_t ld, int64_t col0, uint64_t seed,
                                            int dist, double lo, double hi, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif /* PONNI_B200_H */
