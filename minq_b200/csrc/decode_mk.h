// Decode megakernel (decode_mk.cu): launch parameters and host helpers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/minq_cuda.h"

namespace minq {

// One projection phase, the same for every layer: rows (gate/up row pairs
// for the dual phase) x cols of 32-column blocks.
struct MkMat {
  int rows;
  int cols;
};

// Per-layer weights and vectors (device array).
struct MkLayerPtrs {
  const uint8_t* w_qkv;   // fused q|k|v blocks [qd + 2 kvd][H]
  const uint8_t* w_o;     // [H][qd]
  const uint8_t* w_gate;  // [I][H]
  const uint8_t* w_up;    // [I][H]
  const uint8_t* w_down;  // [H][I]
  const float* attn_norm;
  const float* ffn_norm;
  const float* bias_qkv;  // may be null
  const float* q_norm;    // may be null
  const float* k_norm;    // may be null
};

static_assert(sizeof(MkLayerPtrs) % 8 == 0, "copied as 8-byte words");

struct MkParams {
  const MkLayerPtrs* layers;   // [n_layers]
  int n_layers;
  MkMat qkv, o, gu, down;
  int H, I, nh, nkv, hd, G, qd, kvd, nsplit, vocab;
  float eps, scale;
  const float* embed;          // [vocab][H] f32
  const float* lm_head;        // tied: == embed
  const float* final_norm;
  const float* rope_cos;       // [max_seq][hd/2]
  const float* rope_sin;
  float* kc;                   // [n_layers][nkv][max_seq][hd]
  float* vc;
  size_t cache_layer_stride;   // nkv * max_seq * hd
  int max_seq;
  float* x;                    // residual stream [H]
  float* qkv_out;              // [qd + 2 kvd]
  float* att;                  // [qd]
  float* h;                    // [I]
  float* logits;               // [vocab]
  float* part;                 // [nkv * nsplit][G][hd + 2]
  unsigned* head_ctr;          // [nkv] monotonic: + history splits per layer
  unsigned* head_base;         // head counters' value at the start of the next launch
  unsigned long long* argmax_part;  // [grid]
  uint32_t* d_tok;             // in: this token; out: its argmax
  int* d_pos;                  // in: history length; out: + 1
  unsigned long long* bar_ctr;   // monotonic grid-barrier counter
  unsigned long long* bar_base;  // counter value at the start of the next launch
  int* status;                 // device status word (bounded-wait timeouts)
  int* abort_flag;             // set when any CTA gives up; every CTA stops
  int want_logits;
  int scratch_bytes;           // x / attention scratch in shared memory
  // The residual stream after the o_proj and down_proj of every layer
  // (exchange sites 2 li and 2 li + 1): [tp_world][H] pairs (value bits,
  // epoch) per site, each row written by one 8-byte store into every rank's
  // slots (tensor parallel: this rank's partial sum, rank 0 adding the
  // residual; one GPU: the row itself). Readers wait until the pairs they
  // need carry this launch's epoch and sum the slots in rank order, so no
  // grid barrier follows o_proj or down_proj.
  int tp_world, tp_rank;
  uint2* const* xr_dst;        // [tp_world]: every rank's pair slots
  const uint2* xr_local;       // this rank's slots [2 n_layers][tp_world][H]
  unsigned* xr_epoch;          // launches so far; this launch's epoch is + 1
};

// The projection plan, or rows == 0 when the consumer's row sums (2 x halves
// x rows per CTA x column warps <= 2048 floats), its column warps (cols / 32
// blocks <= 512, and at most one tile of blocks, so a row spans at most two
// tiles) or its 16-bit block indices do not take the shape.
MkMat mk_plan_mat(int dtype, bool dual, uint64_t rows, uint64_t cols, int grid);
// Shared-memory scratch: the staged input vector, or the attention state
// and one head's split partials for a slice of its outputs.
size_t mk_scratch_bytes(int H, int I, int qd, int G, int hd, int nsplit);
// Shared memory of the launch, or 0 when it does not fit one SM.
size_t mk_smem_bytes(size_t scratch_bytes, int n_layers);
minq_status launch_decode_mk(const MkParams& p, int dtype, int grid, size_t smem,
                             cudaStream_t s);

}  // namespace minq
