// Needle-3 engine on one B200: the GPU counterpart of the reference's
// V3Model + V3Cache + V3Engine (crates/needle-core/src/v3/model.rs,
// v3/cache.rs, crates/needle-infer/src/v3_engine.rs).
#pragma once
#include <cuda_runtime.h>

#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "kernels.hpp"
#include "tokenizer.hpp"

namespace nb {

struct Record {  // crates/needle-infer/src/cact.rs:398-425
  uint8_t dtype = 0, ndim = 0;
  uint32_t shape[4] = {0, 0, 0, 0};
  uint64_t offset = 0, nbytes = 0;
  uint32_t group = 0, bits = 0;
};

struct HostConfig {  // crates/needle-core/src/v3/config.rs:44-73
  size_t vocab = 0, out_vocab = 0, d = 0, heads = 0, kvh = 0, layers = 0, qk = 0, vh = 0,
         max_seq = 0, hada_n = 0, lanes = 0, window = 0, taps = 0;
  std::vector<int> global_layers;
  std::vector<int> orders, sites;
  size_t e_slots = 0, e_sub = 0, e_tables = 0, e_heads = 0, e_taps = 0, e_dil = 0, e_seed_heads = 0;
  float rope_theta = 0.f;
  uint32_t kv_window = 0, kv_bits = 0;
  size_t num_tensors = 0;
  bool has_heads = false;
  size_t logit_rows() const { return out_vocab == 0 ? vocab : out_vocab; }
  bool is_global(size_t l) const;
  size_t span(size_t l) const;  // 0 = unbounded
  size_t kv_bytes_at(size_t seq_len, bool int8) const;  // config.rs:234-272
};

class Engine;

// One generation session: the device-resident counterpart of V3Cache.
class Session {
 public:
  ~Session();
  Engine* eng = nullptr;
  bool int8 = false;
  size_t hint = 0;
  size_t pos = 0;                 // host mirror of SessDesc::pos
  SessDesc* d_desc = nullptr;     // device descriptor
  LayerKV* d_layers = nullptr;    // device array [layers]
  std::vector<LayerKV> layers;    // host mirror
  void* d_state = nullptr;        // tails + token ring (inside the arena)
  void* d_arena = nullptr;        // one allocation holding the initial rings, state and descriptors
  std::vector<char> owned;        // layer ring grown into its own allocation
  uint64_t seen = 0;              // the engine's batch-check stamp of the last call it was in
  // The smallest position at which some layer's ring must grow (its slot count
  // while below its cap); 0 until ensure_slots first computes it, so a step
  // below it skips the per-layer check.
  size_t grow_at = 0;
  size_t state_bytes = 0;
  size_t bytes() const;           // device bytes held, as V3Cache::bytes counts them
};

struct Workspace {
  size_t cap = 0;  // rows
  size_t last_cap = 0;
  float *lanes = nullptr, *u = nullptr, *bx = nullptr, *xh = nullptr, *proj = nullptr,
        *qpost = nullptr, *q8s = nullptr, *oh = nullptr, *projo = nullptr, *gates = nullptr,
        *fetched = nullptr, *ekv = nullptr, *evc = nullptr, *lm_in = nullptr, *pks = nullptr,
        *pvs = nullptr, *logits = nullptr, *lm_last = nullptr;
  void *pk = nullptr, *pv = nullptr;
  int8_t* q8 = nullptr;  // int8 mode: query codes [rows][heads][qk], scales in q8s [rows][heads]
  __half *ahi = nullptr, *alo = nullptr;  // tensor-core projections: split activations
  float* ainv = nullptr;                  // and their inverse group scales [rows][32]
  // The Engram key|value projections' operands, written by the gather in the
  // split form: [sites][rows][d_model] halves, scales [sites][rows][d_model / 128].
  __half *ehi = nullptr, *elo = nullptr;
  float* einv = nullptr;
  // The last forward wrote the LM head's input in the split form (not lm_in).
  bool head_presplit = false;
  __half *whi = nullptr, *wlo = nullptr;  // expanded levels of the projection being computed
  int* cnt = nullptr;  // attention split-arrival counters [rows][kv heads], zero between launches
  unsigned long long* keys = nullptr;  // the LM head's greedy-pick keys [rows] (GemmScratch::amax)
  float* pre_part = nullptr;  // split mHC pre-projection partials [rows][32][32]
  int* pre_cnt = nullptr;     // and its per-row arrival counters, zero between launches
  GemmScratch gs;
  RowInfo* rows = nullptr;
  uint32_t *tokens = nullptr, *next = nullptr;
  int* last_rows = nullptr;
  float* cells = nullptr;  // when set, the forward writes the probe-head cells here [layers + 1][rows][d]
  float* part = nullptr;  // attention split partials
  size_t part_cap = 0;    // floats
  // Pinned host staging of a host-API decode step ([cap] each): the rows and
  // tokens go to the device and the picks come back by DMA, without the
  // driver's pageable-memory staging.
  RowInfo* h_rows = nullptr;
  uint32_t *h_tok = nullptr, *h_pick = nullptr;
  void release();
};

// A fixed set of sessions decoded together. Owns the device array of session
// descriptors and a CUDA graph of one decode step, replayed while the set and
// the ring capacities stay the same.
class Batch {
 public:
  ~Batch();
  Engine* eng = nullptr;
  std::vector<Session*> sessions;
  SessDesc** d_sess = nullptr;
  bool int8 = false;
  cudaGraphExec_t graph = nullptr;
  bool graph_logits = false;
  uint64_t graph_epoch = 0;
  uint64_t warm_epoch = 0;
  int nsplit = 0;              // attention splits baked into the graph
  uint32_t* d_tok = nullptr;   // [n] token fed this step
  uint32_t* d_next = nullptr;  // [n] greedy pick of this step
};

// Kernel groups of one forward, for per-kernel timing.
enum ProfKind {
  PK_ENGRAM = 0, PK_EMBED, PK_LAYER_PRE, PK_QKVG, PK_QKV_POST, PK_ATTN, PK_ATTN_FINISH, PK_OUT_PROJ,
  PK_LAYER_POST, PK_FINAL, PK_HEAD, PK_BOOK, PK_COUNT
};

// Events recorded after each launch group of a step; `launches` counts this
// library's kernel launches.
struct Prof {
  std::vector<std::pair<int, cudaEvent_t>> marks;
  size_t used = 0;
  int launches = 0;
  cudaError_t mark(int kind, cudaStream_t st, int nlaunch);
};

class Engine {
 public:
  // depth 0 (or the container's own depth) loads every block; 2..layers-1
  // loads that rung of the intelligence ladder (v3.rs:656-745).
  static Engine* load(const uint8_t* data, size_t len, std::string* err, size_t depth = 0);
  // One decode step of `b`, eager, with events between kernel groups; writes
  // per-kind milliseconds (PK_COUNT floats) and the number of launches.
  bool profile_batch_step(Batch* b, float* ms, int* launches, std::string* err);
  ~Engine();

  HostConfig cfg;
  Geo G{};
  int device = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  uint64_t batch_stamp = 0;  // per call of a session-list API, under mu: O(n) duplicate checks

  Session* new_session(size_t hint, bool int8, std::string* err);
  // Whole-prompt prefill of fresh sessions (model.rs:512-523). Writes the last
  // position's logits (host, [n][logit_rows]) and/or greedy picks (host, [n]).
  // d_cells: capture the probe-head cells of a single prompt there (device,
  // [layers + 1][len][d_model]).
  bool prefill(Session* const* ss, const uint32_t* const* ids, const size_t* lens, size_t n,
               float* logits, uint32_t* picks, std::string* err, float* d_cells = nullptr);
  // The confidence head's logit over ids (model.rs:482-492); false with *err
  // when the container has no confidence head.
  bool confidence(const uint32_t* ids, size_t n, float* logit, std::string* err);
  // One decode step for each session (model.rs:150-375), host buffers.
  bool decode(Session* const* ss, const uint32_t* tokens, size_t n, float* logits,
              uint32_t* picks, std::string* err);
  // Device-resident decode step over a batch: reads b->d_tok, writes b->d_next
  // and (when logits != nullptr) logits [n][logit_rows] on the device.
  bool decode_batch_device(Batch* b, float* d_logits, cudaStream_t st, bool use_graph,
                           std::string* err);
  Batch* new_batch(Session* const* ss, size_t n, std::string* err);
  // Host copy of layer `li`'s ring in the reference's layout (V3Cache::kv,
  // cache.rs:382-393): k [slots][kv_heads][qk], v [slots][kv_heads][vh], f32
  // or int8 codes by the session's precision, and for int8 the scales
  // [slots][kv_heads]. Synchronous.
  bool read_kv(Session* s, size_t li, void* k, void* v, float* ks, float* vs, std::string* err);

  // --- weights on the device
  uint8_t* d_blob = nullptr;
  float* d_params = nullptr;
  uint32_t* d_perm = nullptr;
  float* d_rope = nullptr;
  uint32_t* d_hfrag = nullptr;  // HadamardMLP weight fragments, all layers
  float* d_phid = nullptr;
  float* d_conf = nullptr;  // the confidence head's weights (conf points into it)
  std::vector<void*> d_owned;  // 3-bit and ternary tensors widened to 4-bit codes
  ProbeHeadDev conf{};
  // The container's tokenizer (its RAW record); null when the container has none.
  std::unique_ptr<Tokenizer> tok;      // mHC lane-matrix rows, dequantised and rotated, all container layers
  CqMat emb{}, phi_pre{}, phi_post{}, phi_res{};
  std::vector<CqMat> qkvg, outp, eng_kv, eng_tables;
  CqMat* d_tables = nullptr;
  std::vector<LayerParams> lp;
  std::vector<MhcParams> mp;
  std::vector<const float*> eng_taps;
  std::vector<int> site_of;
  const float* final_norm = nullptr;
  Workspace ws;
  uint64_t epoch = 1;  // bumped whenever a session's device layout changes
  // Graph of the host-API decode step (forward, step end, head), replayed
  // while the row count, split count, KV precision and epoch are unchanged;
  // the step's rows and tokens are copied in before it, the picks out after.
  cudaGraphExec_t dec_graph = nullptr;
  uint64_t dec_graph_epoch = 0, dec_warm_epoch = 0;
  size_t dec_n = 0;
  int dec_ns = 0, dec_int8 = -1, dec_logits = -1;
  // This engine's own device flag, raised by its tensor-core GEMMs and int8
  // attention when a bounded wait expired; no other handle reads or clears it.
  int* d_wait_flag = nullptr;
  int* h_wait_flag = nullptr;  // pinned host copy, refreshed before each synchronous return

  // Queues the copy of the device wait flag on `st`; after the stream is
  // synchronised, wait_status() turns a raised flag into an error and clears it.
  cudaError_t queue_wait_flag(cudaStream_t st);
  cudaError_t wait_status(cudaStream_t st);
  // Synchronous read of the device flag: cudaErrorTimeout (and the flag
  // cleared) when it was raised.
  cudaError_t take_wait_flag();

  bool ensure_ws(Workspace& w, size_t rows, std::string* err);
  bool ensure_part(Workspace& w, size_t rows, int nsplit, std::string* err);
  bool ensure_slots(Session* s, size_t pos, std::string* err);
  // split_head: every row goes to the LM head next (decode), so the final
  // kernel may write the head's tensor-core operands instead of lm_in.
  cudaError_t forward(Workspace& w, const RowBatch& rb, cudaStream_t st, bool int8, int nsplit,
                      Prof* prof = nullptr, bool split_head = false);
  // need_logits false: only the picks are wanted, and a head on the
  // tensor-core operands the final kernel wrote folds the greedy pick into the
  // projection instead of storing [M][logit_rows] logits.
  cudaError_t head(Workspace& w, const float* lm_in, int ldx, int M, float* logits, uint32_t* picks,
                   cudaStream_t st, Prof* prof = nullptr, bool need_logits = true);
};

}  // namespace nb
