// Host side of the tensor-core dense-chain kernel: eligibility, operand
// packing (the swizzled K-major weight images) and the TcProgram.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "model.h"
#include "tc_plan.h"
#include "tc_resid.h"
#include "tc_stream.h"

namespace ponni_b200 {
namespace {

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

bool tc_activation(int k) {
  return k == PONNI_B200_RELU || k == PONNI_B200_LEAKY_RELU || k == PONNI_B200_SILU || k == PONNI_B200_GELU ||
         k == PONNI_B200_TANH || k == PONNI_B200_SIGMOID;
}

// Place one element into a K-major SW128 operand with `rows` rows.
size_t put_kmajor(std::vector<unsigned char>& img, size_t base, int rows, int n, int k, int esz, const void* val) {
  const int kper = 128 / esz;
  const int kb = k / kper;
  const int wb = (k % kper) * esz;
  const int chunk = wb / 16;
  const size_t off = base + (size_t)kb * rows * 128 + (size_t)n * 128 + (size_t)((chunk ^ (n & 7)) * 16) + (wb % 16);
  memcpy(img.data() + off, val, esz);
  return off;
}

uint32_t make_idesc(int dtype, int n_pad, bool a_mn_major) {
  // fp32 models run on bf16 operand parts
  const uint32_t fmt = dtype == PONNI_B200_F16 ? 0u : 1u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((uint32_t)(n_pad >> 3) << 17) |
         ((uint32_t)(kTcM >> 4) << 24);
}

}  // namespace

bool tc_plan(const ponni_b200_model* m, TcProgram& p, std::vector<unsigned char>& image, std::string& why,
             ParamMap* rec) {
  memset(&p, 0, sizeof(p));
  image.clear();
  const ponni_b200_dtype dt = m->dtype;
  if (dt != PONNI_B200_F32 && dt != PONNI_B200_F16 && dt != PONNI_B200_BF16) {
    why = "tensor-core path supports fp32 (bf16 3-way split), fp16 and bf16 models";
    return false;
  }
  const bool split = dt == PONNI_B200_F32;
  const int nparts = split ? 3 : 1;
  const int kstep = 16;  // UMMA K for 16-bit operands
  const size_t msz = dtype_bytes(dt);
  // Walk [Matvec][Bias]?[activation]? blocks.
  struct Blk { const Layer* mv; const Layer* bias; const Layer* act; };
  std::vector<Blk> blocks;
  const auto& Ls = m->layers;
  for (size_t i = 0; i < Ls.size();) {
    if (Ls[i].d.kind != PONNI_B200_MATVEC) {
      why = std::string("layer ") + layer_label(Ls[i].d.kind) + " is outside a dense chain";
      return false;
    }
    Blk b{&Ls[i], nullptr, nullptr};
    ++i;
    if (i < Ls.size() && Ls[i].d.kind == PONNI_B200_BIAS) b.bias = &Ls[i++];
    if (i < Ls.size() && tc_activation(Ls[i].d.kind)) b.act = &Ls[i++];
    blocks.push_back(b);
  }
  if (blocks.empty() || blocks.size() > (size_t)kTcMaxLayers) {
    why = "dense chain length out of range";
    return false;
  }
  p.n_layers = (int)blocks.size();
  p.dtype = (int)dt;
  p.nparts = nparts;
  p.nin = blocks.front().mv->d.num_inputs;
  p.nout = blocks.back().mv->d.num_outputs;
  int max_npad = 0, max_w32 = 0;
  for (size_t l = 0; l < blocks.size(); ++l) {
    const auto& d = blocks[l].mv->d;
    if (d.num_inputs > 256 || d.num_outputs > 256) {
      why = "layer wider than 256";
      return false;
    }
    TcLayer& L = p.layers[l];
    L.nin = d.num_inputs;
    L.nout = d.num_outputs;
    L.k_pad = (int)round_up(d.num_inputs, kstep);
    L.n_pad = (int)round_up(d.num_outputs, 16);
    L.act = blocks[l].act ? blocks[l].act->d.kind : EPI_NONE;
    L.act_flags = blocks[l].act ? blocks[l].act->d.flags : 0;
    L.s0 = blocks[l].act ? (float)blocks[l].act->d.scalar[0] : 0.f;
    L.s1 = blocks[l].act ? (float)blocks[l].act->d.scalar[1] : 0.f;
    L.has_bias = blocks[l].bias ? 1 : 0;
    L.idesc = make_idesc(dt, L.n_pad, false);
    L.idesc_mn = make_idesc(dt, L.n_pad, true);
    if (l + 1 < blocks.size()) max_w32 = std::max(max_w32, (int)round_up(L.n_pad, 32));
  }
  // Image: biases first, then weights at 1024-byte aligned offsets.
  // fp32 (split) models: float biases padded to 32 columns, added in the
  // epilogue.  16-bit models: the bias is one more UMMA of K = 16 whose A is
  // a column of ones and whose B holds the bias in column 0, both in the
  // no-swizzle K-major layout (core matrices of 8 rows x 16 bytes).  Only the
  // first K half (elements 0-7) of each row is stored: the ones block is one
  // core matrix that every row group of A reads (row-group stride 0), a bias
  // block is n_pad / 8 core matrices (row-group stride 128 bytes), and the
  // second K half of both points into one shared block of zeros.  The
  // epilogue then neither loads nor adds the bias.
  size_t off = 0;
  bool any_bias = false;
  for (const auto& b : blocks) any_bias = any_bias || b.bias != nullptr;
  if (!split && any_bias) {
    p.ones_off = 0;
    off = 128;
  }
  int max_np = 0;
  for (int l = 0; l < p.n_layers; ++l) {
    TcLayer& L = p.layers[l];
    L.bias_off = (uint32_t)off;
    if (split) {
      off += round_up(round_up(L.n_pad, 32) * 4, 16);
    } else if (L.has_bias) {
      L.has_bias = 0;
      L.bias_mma = 1;
      off += (size_t)L.n_pad * 16;
      max_np = std::max(max_np, L.n_pad);
    }
  }
  if (!split && any_bias) {
    p.zero_off = (uint32_t)off;
    off += (size_t)max_np * 16;
  }
  off = round_up(off, 1024);
  for (int l = 0; l < p.n_layers; ++l) {
    TcLayer& L = p.layers[l];
    const int nkb = (int)((L.k_pad * 2 + 127) / 128);
    const size_t bytes = (size_t)nkb * L.n_pad * 128;
    for (int q = 0; q < 3; ++q) {
      L.w_off[q] = (uint32_t)off;
      if (q < nparts) off += round_up(bytes, 1024);
    }
  }
  p.image_bytes = (uint32_t)round_up(off, 1024);
  image.assign(p.image_bytes, 0);
  if (!split && any_bias) {
    // ones block: rows 0..7, K = 0 is 1.0 in the model's 16-bit type
    const uint16_t one = dt == PONNI_B200_F16 ? 0x3C00u : 0x3F80u;
    for (int r = 0; r < 8; ++r) memcpy(image.data() + p.ones_off + (size_t)r * 16, &one, 2);
  }
  for (int l = 0; l < p.n_layers; ++l) {
    const TcLayer& L = p.layers[l];
    const Layer& mv = *blocks[l].mv;
    if (blocks[l].bias && split) {
      float* b = reinterpret_cast<float*>(image.data() + L.bias_off);
      for (int f = 0; f < L.nout; ++f) {
        b[f] = (float)load_scalar(dt, blocks[l].bias->params.data() + f * msz);
        if (rec) rec->add(blocks[l].bias->params.data() + f * msz, PIMG_TC, PENC_F32, L.bias_off + 4 * (size_t)f);
      }
    } else if (blocks[l].bias) {
      // bias[n] at K = 0 of row n: row group n / 8, row n % 8 of its core matrix
      for (int f = 0; f < L.nout; ++f) {
        const size_t o = L.bias_off + (size_t)(f >> 3) * 128 + (size_t)(f & 7) * 16;
        memcpy(image.data() + o, blocks[l].bias->params.data() + f * msz, msz);
        if (rec) rec->add(blocks[l].bias->params.data() + f * msz, PIMG_TC, PENC_MODEL, o);
      }
    }
    for (int k = 0; k < L.nin; ++k) {
      for (int n = 0; n < L.nout; ++n) {
        const unsigned char* src = mv.params.data() + ((size_t)k * L.nout + n) * msz;  // W[k][n]
        if (split) {
          float w;
          memcpy(&w, src, 4);
          // exact three-way bf16 split w = b0 + b1 + b2
          const __nv_bfloat16 b0 = __float2bfloat16_rn(w);
          const float r = w - __bfloat162float(b0);
          const __nv_bfloat16 b1 = __float2bfloat16_rn(r);
          const __nv_bfloat16 b2 = __float2bfloat16_rn(r - __bfloat162float(b1));
          const size_t o0 = put_kmajor(image, L.w_off[0], L.n_pad, n, k, 2, &b0);
          const size_t o1 = put_kmajor(image, L.w_off[1], L.n_pad, n, k, 2, &b1);
          const size_t o2 = put_kmajor(image, L.w_off[2], L.n_pad, n, k, 2, &b2);
          if (rec) {
            rec->add(src, PIMG_TC, PENC_SPLIT0, o0);
            rec->add(src, PIMG_TC, PENC_SPLIT1, o1);
            rec->add(src, PIMG_TC, PENC_SPLIT2, o2);
          }
        } else {
          const size_t o = put_kmajor(image, L.w_off[0], L.n_pad, n, k, 2, src);
          if (rec) rec->add(src, PIMG_TC, PENC_MODEL, o);
        }
      }
    }
  }
  const int k0 = p.layers[0].k_pad;
  if (split) max_w32 = std::max(max_w32, (int)round_up(k0, 32));  // fp32 layer 0 is K-major
  // 16-bit: the staged input is the MN-major layer-0 operand (k0/8 atoms of 2 KB).
  p.stage_bytes = split ? 0u : (uint32_t)(k0 / 8) * 2048;  // fp32: input read straight into the split
  const uint32_t a_kmajor = (uint32_t)((max_w32 * 2 + 127) / 128) * kTcM * 128;
  p.a_bytes = std::max(a_kmajor, 1024u);
  p.slot_bytes = p.a_bytes * (uint32_t)nparts + p.stage_bytes;
  // As many tile slots (tiles in flight per SM) as shared and tensor memory
  // allow.  fp32 (split) models use ceil(steps / gs) main accumulators of
  // the dominant products (PONNI_B200_TC_GROUP_STEPS K steps each; default 4)
  // plus one accumulator of the smaller products, summed in the epilogue: the
  // tensor core's fp32 accumulation truncates, so short chains into each main
  // accumulator keep the result fp32-accurate; a slot count that would force
  // longer chains is skipped unless nothing else fits.
  int gs_req = 4;
  if (const char* env = getenv("PONNI_B200_TC_GROUP_STEPS")) gs_req = std::max(1, atoi(env));
  for (int pass = 0; pass < 2; ++pass) {
    for (int slots = kTcMaxSlots; slots >= 1; --slots) {
      // 128-thread slots: up to 8 for 16-bit models (64 registers a thread),
      // up to 4 for fp32 split models (their epilogue needs 128 registers)
      if (slots * (slots >= 3 ? 128 : 256) > (split ? kTcMaxThreads / 2 : kTcMaxThreads)) continue;
      const int col_budget = 512 / slots;
      max_npad = 0;
      bool longer = false;
      for (int l = 0; l < p.n_layers; ++l) {
        TcLayer& L = p.layers[l];
        const int nsteps = L.k_pad / 16;
        const int extra = split ? 1 : 0;  // the correction accumulator
        int gs = split ? std::min(gs_req, nsteps) : nsteps;
        while (gs < nsteps && round_up((int64_t)((nsteps + gs - 1) / gs + extra) * L.n_pad, 32) > col_budget) ++gs;
        if (split && gs > gs_req && gs < nsteps) longer = true;
        L.group_steps = std::min(gs, nsteps);
        L.groups = (nsteps + L.group_steps - 1) / L.group_steps + extra;
        max_npad = std::max(max_npad, L.groups * L.n_pad);
      }
      if (longer && pass == 0) continue;
      p.slot_cols = (uint32_t)round_up(max_npad, 32);
      uint32_t cols = 32;
      while (cols < (uint32_t)slots * p.slot_cols) cols <<= 1;
      p.smem_bytes = 1024 + p.image_bytes + (uint32_t)slots * p.slot_bytes + 128 +
                     (uint32_t)(kTcMaxLayers * sizeof(TcLayer));
      if (cols <= 512 && p.smem_bytes <= 227 * 1024) {
        p.tmem_cols = cols;
        p.slots = slots;
        p.slot_threads = slots >= 3 ? 128 : 256;
        return true;
      }
    }
  }
  why = "weights and operand tiles exceed shared memory";
  return false;
}

bool ts_plan(const ponni_b200_model* m, TsProgram& p, std::vector<unsigned char>& image, std::string& why,
             ParamMap* rec) {
  memset(&p, 0, sizeof(p));
  image.clear();
  const ponni_b200_dtype dt = m->dtype;
  if (dt != PONNI_B200_F16 && dt != PONNI_B200_BF16) {
    why = "the streamed tensor-core path supports fp16 and bf16 models";
    return false;
  }
  const size_t msz = dtype_bytes(dt);
  struct Blk { const Layer* mv; const Layer* bias; const Layer* act; };
  std::vector<Blk> blocks;
  const auto& Ls = m->layers;
  for (size_t i = 0; i < Ls.size();) {
    if (Ls[i].d.kind != PONNI_B200_MATVEC) {
      why = std::string("layer ") + layer_label(Ls[i].d.kind) + " is outside a dense chain";
      return false;
    }
    Blk b{&Ls[i], nullptr, nullptr};
    ++i;
    if (i < Ls.size() && Ls[i].d.kind == PONNI_B200_BIAS) b.bias = &Ls[i++];
    if (i < Ls.size() && tc_activation(Ls[i].d.kind)) b.act = &Ls[i++];
    blocks.push_back(b);
  }
  if (blocks.empty() || blocks.size() > (size_t)kTsMaxLayers) {
    why = "dense chain length out of range";
    return false;
  }
  p.n_layers = (int)blocks.size();
  p.dtype = (int)dt;
  p.fast_act = 1;
  p.nin = blocks.front().mv->d.num_inputs;
  p.nout = blocks.back().mv->d.num_outputs;
  uint64_t off = 0;
  uint32_t a_blocks = 1;
  for (int l = 0; l < p.n_layers; ++l) {
    const auto& d = blocks[l].mv->d;
    if (d.num_inputs > kTsMaxN || d.num_outputs > kTsMaxN) {
      why = "layer wider than 256";
      return false;
    }
    TsLayer& L = p.layers[l];
    L.nin = d.num_inputs;
    L.nout = d.num_outputs;
    L.k_pad = (int)round_up(d.num_inputs, 16);
    L.n_pad = (int)round_up(d.num_outputs, 16);
    L.kblk = (L.k_pad + kTsBlockK - 1) / kTsBlockK;
    L.act = blocks[l].act ? blocks[l].act->d.kind : EPI_NONE;
    L.act_flags = blocks[l].act ? blocks[l].act->d.flags : 0;
    L.s0 = blocks[l].act ? (float)blocks[l].act->d.scalar[0] : 0.f;
    L.s1 = blocks[l].act ? (float)blocks[l].act->d.scalar[1] : 0.f;
    L.has_bias = blocks[l].bias ? 1 : 0;
    L.w_off = off;
    off += (uint64_t)L.kblk * kTsChunkBytes;
    if (l + 1 < p.n_layers) a_blocks = std::max(a_blocks, (uint32_t)((L.n_pad + 63) / 64));
  }
  for (int l = 0; l < p.n_layers; ++l) {
    p.layers[l].bias_off = (uint32_t)off;
    off += (uint64_t)round_up(round_up(p.layers[l].n_pad, 32) * 4, 16);
  }
  p.image_bytes = round_up((int64_t)off, 1024);
  image.assign(p.image_bytes, 0);
  for (int l = 0; l < p.n_layers; ++l) {
    const TsLayer& L = p.layers[l];
    const Layer& mv = *blocks[l].mv;
    if (blocks[l].bias) {
      float* b = reinterpret_cast<float*>(image.data() + L.bias_off);
      for (int f = 0; f < L.nout; ++f) {
        b[f] = (float)load_scalar(dt, blocks[l].bias->params.data() + f * msz);
        if (rec) rec->add(blocks[l].bias->params.data() + f * msz, PIMG_TS, PENC_F32, L.bias_off + 4 * (size_t)f);
      }
    }
    for (int n = 0; n < L.nout; ++n)
      for (int k = 0; k < L.nin; ++k) {
        const size_t chunk = L.w_off + (size_t)(k / kTsBlockK) * kTsChunkBytes;
        const unsigned char* src = mv.params.data() + ((size_t)k * L.nout + n) * msz;
        const size_t o = put_kmajor(image, chunk, L.n_pad, n, k % kTsBlockK, 2, src);
        if (rec) rec->add(src, PIMG_TS, PENC_MODEL, o);
      }
  }
  p.stage_bytes = (uint32_t)(p.layers[0].k_pad / 8) * 2048;
  p.a_bytes = std::max(a_blocks * (uint32_t)(kTcM * 128), (p.stage_bytes + 1023u) & ~1023u);
  const uint32_t fixed = 1024 + kTsSlots * p.a_bytes + kTsBarBytes + (uint32_t)(kTsMaxLayers * sizeof(TsLayer));
  const uint32_t budget = 227 * 1024;
  // CTA pairs (M = 256 over two SMs, each staging half of every chunk) with
  // PONNI_B200_TS_PAIR=1.  Off by default: on the 64->256x5->32 bf16 chain
  // the pair is slower (148.6 against 126.2 ms per 2^27 columns), because the
  // single CTA's MMA issue already runs at tensor-pipe speed and the pair
  // couples two epilogues and adds a relay hop to every weight stage.
  const char* pe = getenv("PONNI_B200_TS_PAIR");
  p.pair = (pe && atoi(pe) == 1) ? 1 : 0;
  const uint32_t stage = p.pair ? kTsChunkBytes / 2 : kTsChunkBytes;
  if (fixed + 2 * stage > budget) {
    why = "operand tiles exceed shared memory";
    return false;
  }
  p.ring_stages = std::min<uint32_t>(kTsMaxStages, (budget - fixed) / stage);
  p.smem_bytes = fixed + p.ring_stages * stage;
  return true;
}

// Residual / LayerNorm chains (tc_resid.cu): one job per Matvec, every
// layer up to the next Matvec lowered to the job's epilogue operations.
bool tr_plan(const ponni_b200_model* m, TrProgram& p, std::vector<unsigned char>& image, std::string& why,
             ParamMap* rec) {
  memset(&p, 0, sizeof(p));
  image.clear();
  const ponni_b200_dtype dt = m->dtype;
  if (dt != PONNI_B200_F32) {
    why = "the residual tensor-core path supports fp32 models (bf16 3-way split)";
    return false;
  }
  const size_t msz = dtype_bytes(dt);
  const auto& Ls = m->layers;
  if (Ls.empty() || Ls[0].d.kind != PONNI_B200_MATVEC) {
    why = "the chain must start with a Matvec";
    return false;
  }
  int save_slot_of[64];
  for (int& v : save_slot_of) v = -1;
  std::vector<std::pair<int, const Layer*>> vec_ops;  // (op index, layer) of BIAS and LN operations
  int nl = 0, nops = 0;
  for (size_t i = 0; i < Ls.size();) {
    const auto& d = Ls[i].d;
    if (d.kind != PONNI_B200_MATVEC) {
      why = std::string("layer ") + layer_label(d.kind) + " cannot start a dense job";
      return false;
    }
    if (nl == kTrMaxLayers) {
      why = "too many Matvec layers";
      return false;
    }
    if (d.num_inputs > kTrMaxN || d.num_outputs > kTrMaxN) {
      why = "layer wider than 128";
      return false;
    }
    TrLayer& L = p.layers[nl];
    L.nin = d.num_inputs;
    L.nout = d.num_outputs;
    L.k_pad = (int)round_up(L.nin, 16);
    L.n_pad = (int)round_up(L.nout, 16);
    L.kblk = (L.k_pad + 63) / 64;
    L.nsteps = L.k_pad / 16;
    L.op_first = nops;
    L.ln = -1;
    L.idesc = make_idesc(dt, L.n_pad, false);
    // Accumulators: groups of one K block (four K steps) of the dominant
    // products where the job's 128 accumulator columns allow, else one
    // group; the smaller products go into group 0 before its x0*w0 steps.
    int gs = std::min(4, L.nsteps);
    if ((int64_t)((L.nsteps + gs - 1) / gs) * L.n_pad > (int64_t)kTrAccCols) gs = L.nsteps;
    L.group_steps = gs;
    L.groups = (L.nsteps + gs - 1) / gs;
    ++i;
    for (; i < Ls.size() && Ls[i].d.kind != PONNI_B200_MATVEC; ++i) {
      const auto& e = Ls[i].d;
      if (nops == kTrMaxOps) {
        why = "too many epilogue layers";
        return false;
      }
      if (e.num_inputs != L.nout && e.kind != PONNI_B200_BIAS) {
        why = std::string("layer ") + layer_label(e.kind) + " changes the width inside an epilogue";
        return false;
      }
      TrOp& o = p.ops[nops];
      o.flags = e.flags;
      o.s0 = (float)e.scalar[0];
      o.s1 = (float)e.scalar[1];
      if (e.kind == PONNI_B200_BIAS) {
        if (e.num_outputs != L.nout) {
          why = "Bias width differs from the Matvec output";
          return false;
        }
        o.kind = TR_BIAS;
        vec_ops.push_back({nops, &Ls[i]});
      } else if (e.kind >= PONNI_B200_RELU && e.kind <= PONNI_B200_MISH) {
        o.kind = TR_ACT;
        o.arg = e.kind;
      } else if (e.kind == PONNI_B200_SAVE_STATE || e.kind == PONNI_B200_BINOP_ADD) {
        if (e.save_index < 0 || e.save_index >= 64) {
          why = "saved-state index out of range";
          return false;
        }
        int& slot = save_slot_of[e.save_index];
        if (e.kind == PONNI_B200_SAVE_STATE && slot < 0) {
          if (p.n_saved == kTrMaxSaved) {
            why = "more than two saved states";
            return false;
          }
          slot = p.n_saved++;
        }
        if (slot < 0) {
          why = "Binop_Add of a state that was not saved";
          return false;
        }
        o.kind = e.kind == PONNI_B200_SAVE_STATE ? TR_SAVE : TR_ADD;
        o.arg = slot;
      } else if (e.kind == PONNI_B200_LAYER_NORM) {
        if (L.ln >= 0) {
          why = "two LayerNorms between Matvecs";
          return false;
        }
        o.kind = TR_LN;
        L.ln = nops - L.op_first;
        vec_ops.push_back({nops, &Ls[i]});
      } else {
        why = std::string("layer ") + layer_label(e.kind) + " is not supported by the residual tensor-core path";
        return false;
      }
      ++nops;
    }
    L.n_ops = nops - L.op_first;
    ++nl;
  }
  for (int l = 0; l + 1 < nl; ++l)
    if (p.layers[l].nout != p.layers[l + 1].nin) {
      why = "Matvec widths do not chain";
      return false;
    }
  p.n_layers = nl;
  p.dtype = (int)dt;
  p.nparts = 3;
  p.nin = p.layers[0].nin;
  p.nout = p.layers[nl - 1].nout;
  // Image: per layer the weight chunks of n_pad rows x 128 B (SW128
  // K-major) in the order the MMAs consume them: parts 2 and 1 of each K
  // block, then part 0 of each K block; then the float vectors (bias[128]
  // or gamma[128] beta[128]).
  uint64_t off = 0;
  for (int l = 0; l < nl; ++l) {
    p.layers[l].w_off = off;
    off += (uint64_t)p.layers[l].kblk * 3 * (uint64_t)p.layers[l].n_pad * 128;
  }
  for (auto& v : vec_ops) {
    p.ops[v.first].off = (uint32_t)off;
    off += p.ops[v.first].kind == TR_LN ? 1024 : 512;
  }
  p.image_bytes = (uint64_t)round_up((int64_t)off, 1024);
  image.assign(p.image_bytes, 0);
  for (int l = 0; l < nl; ++l) {
    const TrLayer& L = p.layers[l];
    // The l-th Matvec of the tuple.
    const Layer* mv = nullptr;
    for (int i = 0, c = 0; i < (int)Ls.size(); ++i)
      if (Ls[i].d.kind == PONNI_B200_MATVEC && c++ == l) {
        mv = &Ls[i];
        break;
      }
    const size_t chunk = (size_t)L.n_pad * 128;
    for (int k = 0; k < L.nin; ++k)
      for (int n = 0; n < L.nout; ++n) {
        const unsigned char* src = mv->params.data() + ((size_t)k * L.nout + n) * msz;  // W[k][n]
        float w;
        memcpy(&w, src, 4);
        const __nv_bfloat16 b0 = __float2bfloat16_rn(w);
        const float r = w - __bfloat162float(b0);
        const __nv_bfloat16 b1 = __float2bfloat16_rn(r);
        const __nv_bfloat16 b2 = __float2bfloat16_rn(r - __bfloat162float(b1));
        const size_t kb = (size_t)(k / 64);
        const size_t o2 = put_kmajor(image, L.w_off + (2 * kb + 0) * chunk, L.n_pad, n, k % 64, 2, &b2);
        const size_t o1 = put_kmajor(image, L.w_off + (2 * kb + 1) * chunk, L.n_pad, n, k % 64, 2, &b1);
        const size_t o0 = put_kmajor(image, L.w_off + (2 * (size_t)L.kblk + kb) * chunk, L.n_pad, n, k % 64, 2, &b0);
        if (rec) {
          rec->add(src, PIMG_TS, PENC_SPLIT0, o0);
          rec->add(src, PIMG_TS, PENC_SPLIT1, o1);
          rec->add(src, PIMG_TS, PENC_SPLIT2, o2);
        }
      }
  }
  for (auto& v : vec_ops) {
    const TrOp& o = p.ops[v.first];
    const Layer& L = *v.second;
    float* f = reinterpret_cast<float*>(image.data() + o.off);
    const int n = L.d.num_outputs;
    const int nvec = o.kind == TR_LN ? 2 : 1;  // LayerNorm: gamma then beta
    for (int q = 0; q < nvec; ++q)
      for (int i = 0; i < n; ++i) {
        const unsigned char* src = L.params.data() + ((size_t)q * n + i) * msz;
        f[q * 128 + i] = (float)load_scalar(dt, src);
        if (rec) rec->add(src, PIMG_TS, PENC_F32, o.off + 4 * ((size_t)q * 128 + i));
      }
  }
  // One saved state fits in TMEM beside each slot's accumulators; two go to
  // the global scratch area.
  p.saved_tmem = p.n_saved <= 1 ? 1 : 0;
  p.scratch_per_cta = p.saved_tmem ? 0 : (uint64_t)kTrSlots * (uint64_t)p.n_saved * kTrMaxN * 128 * 4;
  // Shared memory: per slot three operand parts of 2 K blocks, the weight
  // ring, the LayerNorm exchange and the mbarriers.  The dynamic shared
  // memory base is 1024-byte aligned (checked by the kernel), so no slack.
  p.smem_bytes = kTrSlots * 3 * kTrPartBytes + kTrStages * kTrChunkBytes + 128;
  if (p.smem_bytes > 227 * 1024) {
    why = "operand tiles exceed shared memory";
    return false;
  }
  return true;
}

}  // namespace ponni_b200
