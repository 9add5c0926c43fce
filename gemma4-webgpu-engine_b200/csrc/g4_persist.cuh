// The persistent B=1 decode step (g4_persist.cu): the phase list the host builds from the step
// order and the launcher.
#pragma once
#include "g4_kernels.cuh"

namespace g4 {

enum PKind : int { PK_EMBED = 1, PK_DENSE = 2, PK_COMBINE = 3, PK_GEMV = 4, PK_ATTN = 5, PK_ARGMAX = 6 };

// The GEMV phases of a decode step (weight bits, row split, prologue, epilogue).
enum PVariant : int {
  PV_Q0 = 1,      // int4, q/k/v of layer 0: norm prologue
  PV_QKV,         // int4, q/k/v: join prologue
  PV_O1,          // int4, o_proj (x prologue)
  PV_O2,          // int4, o_proj of a global layer (x prologue)
  PV_GATEUP,      // int4, gate/up pair, gelu codes
  PV_DOWN,        // int4, down_proj from codes
  PV_PLEG,        // int8, per_layer_gate: norm-residual prologue, gelu codes
  PV_PLEP,        // int8, per_layer_projection from codes
  PV_HEAD,        // int4, lm_head: join prologue, softcap + argmax partials
};

struct PEmbed {
  const int32_t *tokens;
  const uint8_t *embed_w; const uint16_t *embed_s; float embed_scale;
  const uint8_t *const *ple_slices; int ple_rps; const uint16_t *ple_s;
  int H, ple_cols, ple_group;
  float *residual, *ple_id;
};
struct PDense { const uint16_t *w; const float *x; float *y; int N, K; float alpha; };
struct PCombine { const float *proj, *identity, *gain; float *out; int groups, group_dim; float eps, scale; };
struct PArgmax {
  const float *part_val; const int32_t *part_idx; int n_parts;
  int32_t *token_dev, *token_out; float *value_out; int32_t *pos; int advance;
};

struct PPhase {
  int kind, variant, bits, rs, sync_after;
  GemvArgs g;       // partitioned for the persistent grid
  AttnDec at;       // one column
  PEmbed em;
  PDense de;
  PCombine co;
  PArgmax am;
};

cudaError_t launch_decode_persist(const PPhase *ph, int nph, unsigned *bar, int grid, cudaStream_t st);
// The grid the kernel runs on (one CTA per SM), 0 when it cannot be resident.
int persist_max_grid(int device);
int persist_slot_bytes();
int persist_max_rows();
int persist_error_take();
#ifdef G4_TRACE
int persist_trace_take(unsigned long long *out, int max_records);
#endif

}  // namespace g4
