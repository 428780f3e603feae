// Host-side launch interface of the Needle-3 B200 kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <vector>

#include "common.cuh"

namespace nb {

// Model geometry as the kernels need it (crates/needle-core/src/v3/config.rs).
struct Geo {
  int d, heads, kvh, qk, vh, layers, lanes, hada_n, ba, bb, taps, window, max_seq, vocab, logit_rows;
  int q_dim, k_dim, v_dim, o_dim, qkv_dim, proj_dim;
  int e_tables, e_heads, e_slots, e_sub, e_taps, e_dil, e_maxorder, e_reach, e_stride, n_orders, n_sites;
  int orders[4];
  int cond_rank;
  float embed_scale;
};

// f32 parameters of one layer, widened from the container's FP16 records.
struct LayerParams {
  const float *norm_in, *q_taps, *k_taps, *v_taps, *q_norm, *k_norm, *post_norm, *pre_hada;
  float attn_gate;
  const float *d1, *d2, *b2, *d3, *d4, *w1a, *w1b, *w2a, *w2b, *w3a, *w3b, *cond_v, *cond_u;
  int window;  // attention span, 0 = unbounded (config.rs:216)
  // HadamardMLP weight fragments for the tensor-core tail (B^T and A^T of the
  // three Kronecker pairs, high parts and remainders in mma lane order) and
  // their inverse power-of-two scales; null when the factors are not square
  // 16x16 or 32x32.
  const uint32_t* hfrag;
  float hinv[6];
};

// A probe head's dense weights on the device (heads.rs:41-62): probes
// [cells * probes_per_cell][d], gain [cells * probes_per_cell], query
// [queries][d], row_bias [queries][cells * probes_per_cell], proj
// [out_dim][queries * d], bias [out_dim].
struct ProbeHeadDev {
  const float *probes, *gain, *query, *row_bias, *proj, *bias;
  int cells, probes_per_cell, queries, out_dim;
};

// Longest causal QKV conv the GPU path runs (the shipped geometry has 3 taps).
constexpr int MAX_QKV_TAPS = 4;

struct MhcParams {
  float a_pre, a_post, a_res;
  const float *b_pre, *b_post, *b_res;  // this layer's slices
  // Layer whose rows of the mHC lane matrices this block reads: the block's
  // own index, or its index in the full stack for a ladder rung sliced at
  // load (v3.rs:656-745; the active lane still follows the sliced index).
  int phi_layer;
  // This block's 2n + n^2 rows of the lane matrices, dequantised and rotated
  // per 128-group at load: [2n + n^2][lanes * d_model] f32 (tiled path).
  const float* phi_dense;
};

enum RowMode { MODE_DECODE = 0, MODE_PREFILL = 1 };

struct RowBatch {
  RowInfo* rows;            // [M] device
  const uint32_t* tokens;   // [M] device: token fed at each row
  int M;
  int mode;
};

// Scratch of the tensor-core path (16-byte aligned): the activations split
// into f16 high parts and remainders ([M][in_pad]), `elems` (>= M * in_pad)
// halves each, and the inverse scale of every 128-wide group ([M][in_pad /
// 128]), room for `rows` (>= M) rows of them.
struct GemmScratch {
  __half* hi = nullptr;
  __half* lo = nullptr;
  float* inv = nullptr;
  size_t elems = 0;
  size_t rows = 0;
  // The weight rows' levels expanded to f16 high parts and remainders,
  // `welems` (>= nrows * in_pad) halves each.
  __half* whi = nullptr;
  __half* wlo = nullptr;
  size_t welems = 0;
  // Device flag the GEMM raises when one of its bounded waits gives up; null
  // for the library-wide flag that umma_take_error reads.
  int* werr = nullptr;
  // Greedy pick instead of outputs (tensor-core path only): when set, the
  // projection stores nothing and folds each row's outputs into amax[row] by
  // atomicMax of argmax_key (the row's keys zeroed beforehand); the first
  // maximum's column is then argmax_pick(amax[row]).
  unsigned long long* amax = nullptr;
};

// force_path: 0 automatic (GEMV for M <= 8, else the tensor cores when `gs`
// holds enough scratch, else the SIMT GEMM), 1 GEMV, 2 SIMT GEMM, 3 tensor
// cores; for M <= 8, 4 the SIMT GEMV kernels and 5 the tensor-core GEMV
// (f16-exact levels only).
// presplit: the tensor-core path's operands are already in gs->hi / lo / inv
// (the kernel that produced the rows wrote them, see SplitOut): no split and,
// with levels cached at load, no preparation launch; only for a call that
// cq_umma_takes.
cudaError_t cq_project(const CqMat& W, const float* xh, int ldx, int M, float* y, int ldy, int row0,
                       int nrows, cudaStream_t st, int force_path = 0, const GemmScratch* gs = nullptr,
                       bool presplit = false);
bool umma_supported(const CqMat& W);
// True when cq_project with force_path 0 runs these M rows of W on the tensor
// cores with the scratch gs.
bool cq_umma_takes(const CqMat& W, int M, const GemmScratch* gs);
// Expands every row's levels to the f16 tiles the tensor-core projection reads
// (W->lvl_hi / lvl_lo), once, for a matrix the engine keeps; the buffers are
// appended to `owned` for the caller to free. A matrix the tensor cores cannot
// take is left as it is.
cudaError_t umma_cache_levels(CqMat* W, std::vector<void*>* owned, cudaStream_t st);
// Kernel launches cq_project makes for these arguments (on the tensor-core
// path the GEMM plus, unless presplit with cached levels, the preparation).
int cq_launches(const CqMat& W, int M, const GemmScratch* gs, int force_path = 0, bool presplit = false);
cudaError_t cq_project_umma(const CqMat& W, const float* xh, int ldx, int M, float* y, int ldy, int row0,
                            int nrows, cudaStream_t st, const GemmScratch& gs, bool presplit = false);
// Reads and clears the library-wide device flag raised when a bounded wait of
// the tensor-core GEMM expired and the caller gave no flag of its own
// (GemmScratch::werr null) (*flag != 0).
cudaError_t umma_take_error(int* flag);
// Device address of that library-wide flag on the current device.
cudaError_t umma_error_ptr(int** p);

cudaError_t launch_cq_prepare(const float* x, int M, int in_feat, float* xh, int ld_out,
                              cudaStream_t st);

cudaError_t launch_embed(const Geo& G, const CqMat& emb, const RowBatch& rb, float* lanes,
                         cudaStream_t st);
// so: when set, the fetched rows go out only in the tensor-core operand form of
// the Engram key|value projections, site s at so.hi / lo + s * M * d_model and
// so.inv + s * M * (d_model / 128) (each a [M][d_model] split matrix), instead
// of f32 into `fetched`.
cudaError_t launch_engram_gather(const Geo& G, const CqMat* tables, const RowBatch& rb,
                                 float* fetched, cudaStream_t st, SplitOut so = SplitOut{});
cudaError_t launch_engram_conv(const Geo& G, const float* const* taps, const RowBatch& rb,
                               const float* ekv, float* evc, cudaStream_t st);
// Rows up to which launch_layer_pre spreads each row over one CTA per 128-wide
// lane group (the last CTA of a row runs its tail). Measured at 512 rows this
// form took 1.93 ms per decode step against 0.78 for 4-row tiles.
constexpr int PRE_SPLIT_MAX_ROWS = 8;
// split_part / split_cnt (nullable): scratch of that form, PRE_SPLIT_MAX_ROWS
// rows x 32 groups x 32 floats and PRE_SPLIT_MAX_ROWS zero-initialised counters
// (reset by the kernel).
// so.hi non-null: the rotated attention input goes to so (the q|k|v|gate
// projection's tensor-core operands, [M][dpad]) instead of xh.
cudaError_t launch_layer_pre(const Geo& G, int li, const RowBatch& rb, const float* lanes,
                             const CqMat& phi_pre, const CqMat& phi_post, const CqMat& phi_res,
                             const MhcParams& mp, const float* norm_in, int site, const float* ekv,
                             const float* evc, float* u, float* bx, float* xh, float* gates,
                             cudaStream_t st, float* split_part = nullptr, int* split_cnt = nullptr,
                             SplitOut so = SplitOut{});
// In int8 mode q8out / q8s (when non-null) receive the query's int8 codes
// [M][heads][qk] and per-head scales [M][heads].
cudaError_t launch_qkv_post(const Geo& G, int li, const RowBatch& rb, const LayerParams& lp,
                            const float* rope_cs, const float* proj, float* qpost, void* pk,
                            void* pv, float* pks, float* pvs, int8_t* q8out, float* q8s,
                            cudaStream_t st);
// Attention writes per-(row, KV head, split) partials; attn_finish merges the
// splits, applies the output gate and rotates for out_proj.
int attn_nsplit(int rows, int kvh, int max_span);
size_t attn_part_floats(int rows, int heads, int kvh, int vh, int nsplit);
// int8 = 1 runs the tensor-core kernel on the query codes q8 / q8s;
// int8 = 0 the f32 kernel on qpost.
// With proj / oh / cnt (per-row, per-KV-head counters, zero-initialised) and
// attn_fuses_finish(), either kernel also merges the splits, gates and
// rotates into oh, so attn_finish is not launched.
// werr: device flag set to 2 when a bounded wait of the int8 kernel's copies
// expired (required for int8 = 1). so.hi non-null: the rotated output goes to
// so (out_proj's tensor-core operands, [M][opad]) instead of oh.
cudaError_t launch_attention(const Geo& G, int li, const RowBatch& rb, const LayerParams& lp, int nsplit,
                             const float* qpost, const int8_t* q8, const float* q8s, const void* pk,
                             const void* pv, const float* pks, const float* pvs, float* part,
                             cudaStream_t st, int int8, const float* proj, float* oh, int* cnt, int* werr,
                             SplitOut so = SplitOut{});
bool attn_fuses_finish(const Geo& G, int int8);
cudaError_t launch_attn_finish(const Geo& G, const RowBatch& rb, int nsplit, const float* part,
                               const float* proj, float* oh, cudaStream_t st, SplitOut so = SplitOut{});
cudaError_t launch_layer_post(const Geo& G, int li, const RowBatch& rb, const LayerParams& lp,
                              const uint32_t* p1, const uint32_t* p2, const float* projo,
                              const float* u, float* bx, const float* gates, float* lanes,
                              cudaStream_t st);
// Tensor-core block tail (post_kernels.cu) and the host-side fragment builder.
bool hada_tc_supported(int ba, int bb);
size_t hada_frag_words(int D);
void hada_frags(const float* const* mats, int D, uint32_t* out, float* inv);
cudaError_t launch_layer_post_tc(const Geo& G, const RowBatch& rb, const LayerParams& lp, const uint32_t* p1,
                                 const uint32_t* p2, const float* projo, const float* u, float* bx,
                                 const float* gates, float* lanes, cudaStream_t st);
// Cells of the probe heads: out[M][d] = lane 0 of each row (copy0) or the
// mean of its lanes; then one head over a captured cells array [cells][seq][d]
// (r: scratch [cells * probes_per_cell][d]; out: out_dim logits).
cudaError_t launch_lane_mean(const float* lanes, int M, int n, int d, bool copy0, float* out, cudaStream_t st);
cudaError_t launch_probe_head(const float* cells, int seq, int d, const ProbeHeadDev& h, float* r, float* out,
                              cudaStream_t st);

// so.hi non-null: the rotated head input goes to so (the LM head's
// tensor-core operands, [M][dpad]) instead of lm_in.
// keys: when set (with so), each row's greedy-pick key is zeroed for the LM
// head's GemmScratch::amax.
cudaError_t launch_final(const Geo& G, const RowBatch& rb, const float* lanes,
                         const float* final_norm, float* lm_in, cudaStream_t st, SplitOut so = SplitOut{},
                         unsigned long long* keys = nullptr);
cudaError_t launch_argmax(const float* logits, int M, int n, int ld, uint32_t* out, cudaStream_t st);
// out[r] = argmax_pick(keys[r]) for the rows of a projection run with
// GemmScratch::amax.
cudaError_t launch_argmax_keys(const unsigned long long* keys, int M, uint32_t* out, cudaStream_t st);
cudaError_t launch_step_begin(const RowBatch& rb, SessDesc* const* sess, cudaStream_t st);
cudaError_t launch_step_end(const RowBatch& rb, cudaStream_t st);

// Records the text returned by nd_last_error() (msg, or the CUDA error's name).
void nd_record_error(cudaError_t e, const char* msg);

// Standalone int8 quantiser of head vectors (cache.rs:100-106), bit-exact.
cudaError_t launch_kv_quant(const float* x, int rows, int dim, int8_t* q, float* scales,
                            cudaStream_t st);
// Standalone batched decode attention over caller-provided rings
// (attention.rs:300-377): B independent sessions, each with its own [lo, hi].
// `part` is scratch of attn_part_floats(B, heads, kvh, vh, nsplit) floats.
cudaError_t launch_attend_step(const float* q, const void* k, const void* v, const float* ks,
                               const float* vs, int int8, int slots, const int* lo, const int* hi,
                               int B, int heads, int kvh, int qk, int vh, int nsplit, float* part,
                               float* out, cudaStream_t st);

}  // namespace nb
