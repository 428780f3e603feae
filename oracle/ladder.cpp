// TEST INFRASTRUCTURE — the CPU oracle's restatement of the reference's
// intelligence ladder: which blocks a depth rung keeps
// (crates/needle-core/src/v3/ladder.rs:28-74), the row subset of a CQ tensor
// (crates/needle-core/src/cq.rs:151-175) and the load-time slice of a
// full-depth model to a rung (crates/needle-infer/src/v3.rs:620-745). Only the
// tests and the checker paths use it; the GPU engine has its own loader.
#include <algorithm>
#include <cstring>

#include "oracle.hpp"

namespace oracle {

// ladder.rs:28-61: both endpoints, then the midpoint of the widest gap
// between selected blocks, leftmost gap first on ties.
std::vector<size_t> ladder_order(size_t num_layers) {
  if (num_layers == 0) return {};
  if (num_layers == 1) return {0};
  std::vector<size_t> selected = {0, num_layers - 1};
  std::vector<size_t> order = selected;
  while (order.size() < num_layers) {
    std::sort(selected.begin(), selected.end());
    bool found = false;
    size_t best_gap = 0, best_left = 0, best_right = 0;
    for (size_t i = 0; i + 1 < selected.size(); ++i) {
      const size_t left = selected[i], right = selected[i + 1];
      if (right - left <= 1) continue;
      const size_t gap = right - left;
      if (!found || gap > best_gap || (gap == best_gap && left < best_left)) {
        found = true;
        best_gap = gap;
        best_left = left;
        best_right = right;
      }
    }
    if (!found) break;
    const size_t mid = (best_left + best_right) / 2;
    selected.push_back(mid);
    order.push_back(mid);
  }
  return order;
}

// ladder.rs:67-74: the first `depth` blocks of the order, ascending; depths
// outside 2..=num_layers are not deployable.
bool ladder_layer_indices(size_t num_layers, size_t depth, std::vector<size_t>* kept) {
  if (depth < 2 || depth > num_layers) return false;
  std::vector<size_t> order = ladder_order(num_layers);
  kept->assign(order.begin(), order.begin() + depth);
  std::sort(kept->begin(), kept->end());
  return true;
}

// cq.rs:151-175: rows are packed independently, so a subset is a copy.
bool CqWeight::select_rows(const std::vector<size_t>& rows, CqWeight* out) const {
  CqWeight w = *this;
  w.packed.clear();
  w.norms.clear();
  for (size_t r : rows) {
    if (r >= out_feat) return false;
    w.packed.insert(w.packed.end(), packed.begin() + r * row_bytes, packed.begin() + (r + 1) * row_bytes);
    w.norms.insert(w.norms.end(), norms.begin() + r * num_groups, norms.begin() + (r + 1) * num_groups);
  }
  w.out_feat = rows.size();
  *out = std::move(w);
  return true;
}

// v3.rs:620-640 config_at_depth and :656-745 model_from_cact_at_depth, applied
// to a model loaded at full depth: the kept blocks renumbered contiguously,
// global layers and Engram sites following them (an Engram site survives
// exactly when its block does), per-layer mHC scalars taken at the kept
// blocks and the lane matrices cut to their rows. Nothing is re-quantised.
std::string slice_to_depth(V3Model* m, size_t depth) {
  V3Config& c = m->cfg;
  if (depth == c.num_layers) return "";
  std::vector<size_t> kept;
  if (!ladder_layer_indices(c.num_layers, depth, &kept)) return "depth is outside the ladder";
  auto rank = [&](size_t l, size_t* r) {
    auto it = std::find(kept.begin(), kept.end(), l);
    if (it == kept.end()) return false;
    *r = (size_t)(it - kept.begin());
    return true;
  };
  const size_t n = c.mhc_lanes;
  std::vector<size_t> globals;
  for (size_t l : c.global_layers) {
    size_t r;
    if (rank(l, &r)) globals.push_back(r);
  }
  std::vector<size_t> sites;
  std::vector<V3EngramSite> engrams;
  for (size_t s = 0; s < c.engram.sites.size(); ++s) {
    size_t r;
    if (rank(c.engram.sites[s], &r)) {
      sites.push_back(r);
      engrams.push_back(m->engrams[s]);
    }
  }
  std::vector<V3Layer> layers;
  for (size_t l : kept) layers.push_back(m->layers[l]);
  V3Mhc& mh = m->mhc;
  auto take = [&](const std::vector<float>& v, size_t width) {
    std::vector<float> out;
    for (size_t l : kept) out.insert(out.end(), v.begin() + l * width, v.begin() + (l + 1) * width);
    return out;
  };
  auto rows = [&](size_t width) {
    std::vector<size_t> out;
    for (size_t l : kept)
      for (size_t i = l * width; i < (l + 1) * width; ++i) out.push_back(i);
    return out;
  };
  V3Mhc sliced;
  sliced.a_pre = take(mh.a_pre, 1);
  sliced.a_post = take(mh.a_post, 1);
  sliced.a_res = take(mh.a_res, 1);
  sliced.b_pre = take(mh.b_pre, n);
  sliced.b_post = take(mh.b_post, n);
  sliced.b_res = take(mh.b_res, n * n);
  if (!mh.phi_pre.select_rows(rows(n), &sliced.phi_pre) || !mh.phi_post.select_rows(rows(n), &sliced.phi_post) ||
      !mh.phi_res.select_rows(rows(n * n), &sliced.phi_res))
    return "mHC lane row out of range";
  // confidence_head_at_depth (v3.rs:745-787): cells 0 and 1 + each kept block
  // of probes and gain, and the same cells on the middle axis of row_bias.
  if (m->has_confidence) {
    ProbeHead& h = m->confidence;
    const size_t k = h.probes_per_cell, q = h.queries, d = c.d_model, mm = h.cells * k;
    std::vector<size_t> cl = {0};
    for (size_t l : kept) cl.push_back(l + 1);
    std::vector<float> probes, gain, row_bias;
    for (size_t cc : cl) {
      probes.insert(probes.end(), h.probes.begin() + cc * k * d, h.probes.begin() + (cc + 1) * k * d);
      gain.insert(gain.end(), h.gain.begin() + cc * k, h.gain.begin() + (cc + 1) * k);
    }
    for (size_t qi = 0; qi < q; ++qi)
      for (size_t cc : cl)
        row_bias.insert(row_bias.end(), h.row_bias.begin() + qi * mm + cc * k,
                        h.row_bias.begin() + qi * mm + (cc + 1) * k);
    h.probes = std::move(probes);
    h.gain = std::move(gain);
    h.row_bias = std::move(row_bias);
    h.cells = cl.size();
  }
  c.num_layers = depth;
  c.global_layers = globals;
  c.engram.sites = sites;
  m->layers = std::move(layers);
  m->mhc = std::move(sliced);
  m->engrams = std::move(engrams);
  return "";
}

}  // namespace oracle
