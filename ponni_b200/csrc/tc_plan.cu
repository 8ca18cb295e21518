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
  // Image: biases first (float, padded to 32 columns), then weights at
  // 1024-byte aligned offsets.
  size_t off = 0;
  for (int l = 0; l < p.n_layers; ++l) {
    TcLayer& L = p.layers[l];
    L.bias_off = (uint32_t)off;
    off += round_up(round_up(L.n_pad, 32) * 4, 16);
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
  for (int l = 0; l < p.n_layers; ++l) {
    const TcLayer& L = p.layers[l];
    const Layer& mv = *blocks[l].mv;
    if (blocks[l].bias) {
      float* b = reinterpret_cast<float*>(image.data() + L.bias_off);
      for (int f = 0; f < L.nout; ++f) {
        b[f] = (float)load_scalar(dt, blocks[l].bias->params.data() + f * msz);
        if (rec) rec->add(blocks[l].bias->params.data() + f * msz, PIMG_TC, PENC_F32, L.bias_off + 4 * (size_t)f);
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
  const uint32_t fixed = 1024 + kTsSlots * p.a_bytes + 256 + (uint32_t)(kTsMaxLayers * sizeof(TsLayer));
  const uint32_t budget = 227 * 1024;
  if (fixed + 2 * kTsChunkBytes > budget) {
    why = "operand tiles exceed shared memory";
    return false;
  }
  p.ring_stages = std::min<uint32_t>(kTsMaxStages, (budget - fixed) / kTsChunkBytes);
  p.smem_bytes = fixed + p.ring_stages * kTsChunkBytes;
  return true;
}

}  // namespace ponni_b200
