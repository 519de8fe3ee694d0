// Host-side cascade planner: decode-batch block tables -> cascade plan.
//
// The reference builds no plan: ReferenceBackend::decode_batch loops over the
// queries and re-gathers every block of every table
// (crates/dendrite-core/src/attention/backend.rs:206-283), and the scheduler's
// tree_state is dead (crates/dendrite-core/src/scheduler/mod.rs:31-33).
// Shared prefixes are, however, literally shared physical block ids:
// TreeState::fork clones the parent's BlockTable and bumps refcounts
// (crates/dendrite-core/src/tree/state.rs:49-84,
// crates/dendrite-core/src/cache/block_table.rs:97-103), and append allocates
// fresh blocks for the child (state.rs:87-113, cache/pool.rs:76-97). The plan
// is therefore the trie over the batch's block-id sequences, compressed into
// runs ("nodes") that are each read by one contiguous range of queries in DFS
// order. Every node is read once per KV head; its partial attention states are
// merged along each query's root-to-leaf path.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstring>
#include <unordered_map>

#include "dd_internal.h"

namespace dd {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int check_config(const dd_attn_config* cfg) {
  if (!cfg) return fail(DD_ERR_INVALID_ARGUMENT, "config is NULL");
  const int D = cfg->head_dim;
  // Same rules as BatchDecodeKernel::new (batch_decode.rs:31-55).
  if (D != 64 && D != 128 && D != 256)
    return fail(DD_ERR_INVALID_ARGUMENT,
                "unsupported head_dim: " + std::to_string(D) + ", supported: [64, 128, 256]");
  if (cfg->num_qo_heads <= 0 || cfg->num_kv_heads <= 0)
    return fail(DD_ERR_INVALID_ARGUMENT, "head counts must be positive");
  if (cfg->num_qo_heads % cfg->num_kv_heads != 0)
    return fail(DD_ERR_INVALID_ARGUMENT, "num_qo_heads must be divisible by num_kv_heads");
  if (cfg->page_size != kPageSize)
    return fail(DD_ERR_INVALID_ARGUMENT, "page_size must be 16");
  if (cfg->num_pages < 0) return fail(DD_ERR_INVALID_ARGUMENT, "num_pages must be >= 0");
  switch (cfg->kv_dtype) {
    case DD_DTYPE_BF16: case DD_DTYPE_F32: case DD_DTYPE_E4M3: case DD_DTYPE_MXFP8: break;
    case DD_DTYPE_F16: return fail(DD_ERR_NOT_AVAILABLE, "f16 KV pages are not implemented");
    default: return fail(DD_ERR_INVALID_ARGUMENT, "unknown kv_dtype");
  }
  if (cfg->q_dtype != DD_DTYPE_BF16 && cfg->q_dtype != DD_DTYPE_F32)
    return fail(cfg->q_dtype == DD_DTYPE_F16 ? DD_ERR_NOT_AVAILABLE : DD_ERR_INVALID_ARGUMENT,
                "q_dtype must be bf16 or f32");
  if (cfg->gqa_map != DD_GQA_TILED && cfg->gqa_map != DD_GQA_GROUPED)
    return fail(DD_ERR_INVALID_ARGUMENT, "unknown gqa_map");
  return DD_OK;
}

size_t plan_workspace_bytes(const dd_plan* p) {
  const size_t D = (size_t)p->cfg.head_dim;
  const size_t slots = (size_t)p->num_slots;
  return kWsHeaderBytes + align_up(slots * D * sizeof(float), kAlign) +
         align_up(slots * sizeof(float), kAlign);
}

// Which kernel family handles nodes with `rows` query rows per KV head.
static int kind_for(const dd_attn_config& c, const dd_plan_options& o, int64_t rows);

}  // namespace dd

extern "C" int dd_tc_available(void);  // attn_tc.cu

namespace dd {

static int kind_for(const dd_attn_config& c, const dd_plan_options& o, int64_t rows) {
  if (c.kv_dtype == DD_DTYPE_F32 || c.q_dtype != DD_DTYPE_BF16 || c.head_dim > 128)
    return kItemSimple;
  const bool tc = o.use_tensor_cores && c.head_dim == 128 && dd_tc_available();
  if (tc && o.cta_pairs && rows > 256 && c.kv_dtype == DD_DTYPE_BF16) return kItemTc2;
  if (tc && rows >= 128) return kItemTc;
  return kItemMma;
}

static int row_tile_for(int kind) {
  return kind == kItemTc2 ? 512 : kind == kItemTc ? 256 : kind == kItemMma ? 16 : 64;
}

// SMs of the target GPU (B200); only a load-balancing heuristic, so the
// planner needs no device.
constexpr int kPlanSms = 148;

// Cost model of the tcgen05 kernel (measured on B200 at 1965 MHz; only used
// to size split-K chunks and to schedule items onto CTAs): one 128-token
// tile of one 128-row sub-tile (three 128x128x16 products per 16 tokens and
// its softmax) per SM, plus a fixed cost per work item (Q load, pipeline
// fill, epilogue).
static double tc_tile_ns(int kv_dtype) {
  return kv_dtype == DD_DTYPE_BF16 ? 1720.0 : kv_dtype == DD_DTYPE_E4M3 ? 2000.0 : 2200.0;
}
constexpr double kTcItemNs = 3000.0;
// ns of one SM for a tcgen05 item of `npages` pages and `nrows` rows.
static double tc_item_ns(int kv_dtype, int64_t npages, int64_t nrows) {
  const int64_t tiles = (npages + 7) / 8;
  return (double)tiles * (nrows > 128 ? 2 : 1) * tc_tile_ns(kv_dtype) + kTcItemNs;
}
// Split-K chunks of a tcgen05 node so its items take at most cap_ns (at
// least 32 pages a chunk; at most 8 chunks, or enough
// for one item per SM when the node has few row tiles x KV heads, as one KV
// head of a long tree per GPU).
static int64_t tc_chunks(int kv_dtype, int64_t npages, int64_t nrows, int64_t units, double cap_ns) {
  const double item = tc_item_ns(kv_dtype, npages, nrows);
  const int64_t want = cap_ns > 0.0 ? (int64_t)std::ceil(item / cap_ns - 0.05) : 1;
  const int64_t most = std::max<int64_t>(8, (kPlanSms + units - 1) / std::max<int64_t>(units, 1));
  return std::max<int64_t>(1, std::min<int64_t>({want, most, std::max<int64_t>(1, npages / 32)}));
}
// Partial-state bytes the merge moves per ns (write + read, mostly in L2).
constexpr double kMergeBytesPerNs = 5000.0;

// A radix-tree node: a run [off, off + len) of one source table.
struct Run {
  int32_t q, off, len;          // source table and run within it
  int32_t first_child = -1, last_child = -1, next_sibling = -1;
  int32_t ends_head = -1, ends_tail = -1;  // queries whose table ends here
};

// Working buffers of one planning pass. A plan keeps them (and all its
// arrays) across dd_plan_rebuild, so re-planning every decode step reuses
// memory instead of allocating and faulting in fresh pages.
struct PlanScratch {
  std::vector<int32_t> used, end_next, node_k, node_slot0, node_kind, qcount, qcursor;
  std::vector<Run> runs;
  struct Frame {
    int32_t node;   // plan node index (-1 for the root)
    int32_t child;  // next child run to descend into
  };
  std::vector<Frame> stack;
  std::vector<std::pair<int64_t, int32_t>> keys;
  std::vector<double> sim_cost, sim_load;  // tcgen05 chunk-size search
};

static void reset_plan(dd_plan* p) {
  p->nodes.clear();
  p->pages.clear();
  p->query_order.clear();
  p->path_indptr.clear();
  p->path_slots.clear();
  for (auto& v : p->items) v.clear();
  p->num_slots = p->kv_tokens = p->kv_tokens_flat = p->tc_row_tokens = 0;
  for (auto& k : p->kv_tokens_by_kind) k = 0;
  p->max_depth = 0;
  p->causal = false;
  p->qlimit.clear();
  p->tc_ctas = 0;
  p->tc_order.clear();
  p->tc_cta_begin.clear();
  p->device_base = nullptr;
  p->device_id = -1;
  if (!p->scratch) p->scratch = new PlanScratch();
}

// Builds nodes / pages / query_order from the tables.
static int build_nodes(dd_plan* p, const int32_t* indptr, const uint32_t* ids,
                       const int32_t* ntok) {
  const int B = p->batch_size;
  PlanScratch& sc = *p->scratch;
  std::vector<int32_t>& used = sc.used;
  used.assign(B, 0);
  for (int b = 0; b < B; ++b) {
    const int nb = indptr[b + 1] - indptr[b];
    if (nb < 0) return fail(DD_ERR_INVALID_ARGUMENT, "block_indptr must be non-decreasing");
    if (ntok[b] < 0 || (int64_t)ntok[b] > (int64_t)nb * kPageSize)
      return fail(DD_ERR_INVALID_ARGUMENT,
                  "num_tokens[" + std::to_string(b) + "] exceeds its block table");
    used[b] = (ntok[b] + kPageSize - 1) / kPageSize;
    p->kv_tokens_flat += ntok[b];
  }
  // Block ids must be < num_pages (DendriteError::InvalidBlock,
  // crates/dendrite-core/src/error.rs:15-17). Every position of a table is
  // either the first occurrence of a run (checked when the run is created) or
  // equal to such a position, so checking new runs covers all ids.
  const uint32_t num_pages = (uint32_t)p->cfg.num_pages;
  auto check_ids = [&](const uint32_t* x, int n) -> int {
    uint32_t mx = 0;
    for (int i = 0; i < n; ++i) mx = std::max(mx, x[i]);
    if (n > 0 && mx >= num_pages) {
      for (int i = 0; i < n; ++i)
        if (x[i] >= num_pages) return fail(DD_ERR_INVALID_ARGUMENT, "invalid block id: " + std::to_string(x[i]));
    }
    return DD_OK;
  };
  auto valid_of = [&](int b, int i) {
    return (i == used[b] - 1 && ntok[b] % kPageSize) ? ntok[b] % kPageSize : kPageSize;
  };

  if (!p->opts.share_prefixes) {
    // Flat plan: one node per non-empty query, no sharing.
    p->query_order.resize(B);
    for (int b = 0; b < B; ++b) {
      p->query_order[b] = b;
      if (used[b] == 0) continue;
      if (int st = check_ids(ids + indptr[b], used[b])) return st;
      Node n;
      n.q_begin = b;
      n.num_q = 1;
      n.num_tokens = ntok[b];
      n.page_off = (int32_t)p->pages.size();
      n.page_count = used[b];
      n.last_valid = valid_of(b, used[b] - 1);
      for (int i = 0; i < used[b]; ++i) p->pages.push_back(ids[indptr[b] + i]);
      p->nodes.push_back(n);
    }
    p->max_depth = p->nodes.empty() ? 0 : 1;
    return DD_OK;
  }

  // Radix tree over (page id, valid tokens) sequences. A node is a run of
  // positions [off, off + len) of one source table; inserting a table walks
  // runs with plain element compares and splits a run where the tables part.
  std::vector<Run>& runs = sc.runs;
  runs.clear();
  runs.reserve(2 * (size_t)B + 1);
  runs.push_back(Run{-1, 0, 0});
  std::vector<int32_t>& end_next = sc.end_next;
  end_next.assign(B, -1);
  auto key_eq = [&](int qa, int ia, int qb, int ib) {
    return ids[indptr[qa] + ia] == ids[indptr[qb] + ib] && valid_of(qa, ia) == valid_of(qb, ib);
  };
  auto add_end = [&](int32_t n, int32_t b) {
    if (runs[n].ends_tail < 0) runs[n].ends_head = b;
    else end_next[runs[n].ends_tail] = b;
    runs[n].ends_tail = b;
  };
  auto add_child = [&](int32_t n, int32_t c) {
    if (runs[n].last_child < 0) runs[n].first_child = c;
    else runs[runs[n].last_child].next_sibling = c;
    runs[n].last_child = c;
  };
  for (int b = 0; b < B; ++b) {
    int32_t cur = 0;
    int pos = 0;
    for (;;) {
      if (pos == used[b]) {
        add_end(cur, b);
        break;
      }
      int32_t c = runs[cur].first_child;
      while (c >= 0 && !key_eq(runs[c].q, runs[c].off, b, pos)) c = runs[c].next_sibling;
      if (c < 0) {
        if (int st = check_ids(ids + indptr[b] + pos, used[b] - pos)) return st;
        const int32_t nid = (int32_t)runs.size();
        runs.push_back(Run{b, pos, used[b] - pos});
        add_child(cur, nid);
        add_end(nid, b);
        break;
      }
      const Run rc = runs[c];
      const int lim = std::min(rc.len, used[b] - pos);
      int k = 1;
      {
        // Ids first (contiguous compare), then the valid counts, which can
        // differ only at either table's last page.
        const uint32_t* x = ids + indptr[rc.q] + rc.off;
        const uint32_t* y = ids + indptr[b] + pos;
        // Usually the whole run matches (a shared prefix): one compare.
        if (lim > 1 && std::memcmp(x + 1, y + 1, (size_t)(lim - 1) * sizeof(uint32_t)) == 0) {
          k = lim;
        } else {
          while (k + 8 <= lim && std::memcmp(x + k, y + k, 8 * sizeof(uint32_t)) == 0) k += 8;
          while (k < lim && x[k] == y[k]) ++k;
        }
        // Valid counts can differ only at either table's last page.
        for (const int t : {used[rc.q] - 1 - rc.off, used[b] - 1 - pos})
          if (t >= 1 && t < k && valid_of(rc.q, rc.off + t) != valid_of(b, pos + t)) k = t;
      }
      if (k < rc.len) {
        // Split c after k positions: the tail keeps c's children and ends.
        const int32_t tid = (int32_t)runs.size();
        Run tail{rc.q, rc.off + k, rc.len - k};
        tail.first_child = rc.first_child;
        tail.last_child = rc.last_child;
        tail.ends_head = rc.ends_head;
        tail.ends_tail = rc.ends_tail;
        runs.push_back(tail);
        Run& head = runs[c];
        head.len = k;
        head.first_child = head.last_child = tid;
        head.ends_head = head.ends_tail = -1;
      }
      pos += k;
      cur = c;
    }
  }

  // Pre-order DFS: one plan node per run, queries ending at a run emitted
  // before its children's, so each node's queries are a contiguous range.
  p->query_order.reserve(B);
  for (int32_t b = runs[0].ends_head; b >= 0; b = end_next[b]) p->query_order.push_back(b);
  std::vector<PlanScratch::Frame>& stack = sc.stack;
  stack.clear();
  stack.push_back({-1, runs[0].first_child});
  while (!stack.empty()) {
    PlanScratch::Frame& f = stack.back();
    if (f.child >= 0) {
      const int32_t r = f.child;
      f.child = runs[r].next_sibling;
      const Run& rr = runs[r];
      Node n;
      n.parent = f.node;
      n.depth = f.node < 0 ? 0 : p->nodes[f.node].depth + 1;
      n.q_begin = (int32_t)p->query_order.size();
      n.page_off = (int32_t)p->pages.size();
      n.page_count = rr.len;
      const uint32_t* src = ids + indptr[rr.q] + rr.off;
      p->pages.insert(p->pages.end(), src, src + rr.len);
      n.num_tokens = (rr.len - 1) * kPageSize + valid_of(rr.q, rr.off + rr.len - 1);
      n.last_valid = valid_of(rr.q, rr.off + rr.len - 1);
      for (int32_t b = rr.ends_head; b >= 0; b = end_next[b]) p->query_order.push_back(b);
      p->nodes.push_back(n);
      p->max_depth = std::max(p->max_depth, n.depth + 1);
      stack.push_back({(int32_t)p->nodes.size() - 1, rr.first_child});
    } else {
      if (f.node >= 0) {
        Node& n = p->nodes[f.node];
        n.num_q = (int32_t)p->query_order.size() - n.q_begin;
      }
      stack.pop_back();
    }
  }
  return DD_OK;
}

// Schedules the tcgen05 items onto tc_ctas CTAs (one per SM, or the
// plan's tc_sms), longest first onto the least-loaded CTA. The streaming
// kernel, launched after it as a programmatic dependent, starts on the SMs
// left free and takes each tcgen05 CTA's SM when that CTA finishes.
static void schedule_tc(dd_plan* p) {
  p->tc_ctas = 0;
  p->tc_order.clear();
  p->tc_cta_begin.clear();
  const std::vector<WorkItem>& items = p->items[kItemTc];
  const int n = (int)items.size();
  if (n == 0 || p->opts.tc_sms < 0) return;
  const int kv = p->cfg.kv_dtype;
  std::vector<double> cost(n);
  for (int i = 0; i < n; ++i) cost[i] = tc_item_ns(kv, items[i].npages, items[i].nrows & kItemRowsMask);
  // Items are in decreasing size within each node and nodes in decreasing
  // item size, so assigning them in order to the least-loaded CTA is the
  // longest-processing-time rule. Returns the makespan.
  std::vector<std::pair<double, int32_t>> heap;
  std::vector<int32_t> cta(n);
  auto later = [](const std::pair<double, int32_t>& x, const std::pair<double, int32_t>& y) {
    return x.first > y.first || (x.first == y.first && x.second > y.second);
  };
  auto lpt = [&](int K) {
    heap.clear();
    for (int c = 0; c < K; ++c) heap.push_back({0.0, c});
    double span = 0.0;
    for (int i = 0; i < n; ++i) {
      std::pop_heap(heap.begin(), heap.end(), later);
      auto& h = heap.back();
      cta[i] = h.second;
      h.first += cost[i];
      span = std::max(span, h.first);
      std::push_heap(heap.begin(), heap.end(), later);
    }
    return span;
  };
  const int K = std::max(1, std::min({p->opts.tc_sms > 0 ? p->opts.tc_sms : kPlanSms, n, kPlanSms}));
  lpt(K);
  std::vector<int32_t>& begin = p->tc_cta_begin;
  begin.assign((size_t)K + 1, 0);
  for (int i = 0; i < n; ++i) ++begin[cta[i] + 1];
  for (int c = 0; c < K; ++c) begin[c + 1] += begin[c];
  p->tc_order.resize(n);
  std::vector<int32_t> fill(begin.begin(), begin.end() - 1);
  for (int i = 0; i < n; ++i) p->tc_order[fill[cta[i]]++] = i;
  p->tc_ctas = K;
}

static void build_items(dd_plan* p) {
  const dd_attn_config& c = p->cfg;
  const int Hq = c.num_qo_heads, Hkv = c.num_kv_heads, g = Hq / Hkv, D = c.head_dim;
  const double elem = c.kv_dtype == DD_DTYPE_F32 ? 4.0 : c.kv_dtype == DD_DTYPE_BF16 ? 2.0 : 1.0;
  PlanScratch& sc = *p->scratch;
  const size_t N = p->nodes.size();
  const int B = p->batch_size;
  sc.node_k.assign(N, 1);
  sc.node_slot0.assign(N, 0);
  sc.node_kind.assign(N, 0);
  sc.keys.resize(N);
  sc.qcount.assign((size_t)B + 1, 0);  // difference array, then path lengths
  int64_t n_items[kNumItemKinds] = {0, 0, 0, 0};
  // Split-K cap of the scheduled tcgen05 items: the largest node's item
  // time over k = 1, 2, ... chunks, whichever gives the shortest
  // longest-first schedule plus the merge's extra partial states (written
  // and read once more per chunk). Equal items come in whole rounds, so finer
  // chunks only pay when they even out the last round.
  const bool tc_sched = p->opts.tc_sms >= 0;
  double tc_cap_ns = 0.0;
  if (tc_sched && p->opts.max_chunk_pages <= 0) {
    double item_max = 0.0;
    for (size_t ni = 0; ni < N; ++ni) {
      const Node& n = p->nodes[ni];
      const int64_t rows = (int64_t)n.num_q * g;
      if (kind_for(c, p->opts, rows) != kItemTc) continue;
      item_max = std::max(item_max, tc_item_ns(c.kv_dtype, n.page_count, std::min<int64_t>(rows, 256)));
    }
    const int K = p->opts.tc_sms > 0 ? p->opts.tc_sms : kPlanSms;
    double best = 0.0;
    std::vector<double>& cost = sc.sim_cost;
    std::vector<double>& load = sc.sim_load;
    size_t prev_n = 0;
    for (int R : {1, 2, 3, 4, 5, 6, 8, 12, 16, 24}) {
      if (item_max <= 0.0) break;
      const double cap = item_max / R * 1.0001;
      cost.clear();
      double merge_bytes = 0.0;
      for (size_t ni = 0; ni < N; ++ni) {
        const Node& n = p->nodes[ni];
        const int64_t rows = (int64_t)n.num_q * g;
        if (kind_for(c, p->opts, rows) != kItemTc) continue;
        const int64_t k = tc_chunks(c.kv_dtype, n.page_count, std::min<int64_t>(rows, 256),
                                    (rows + 255) / 256 * Hkv, cap);
        merge_bytes += (double)(k - 1) * n.num_q * Hq * (D + 1) * 4.0 * 2.0;
        for (int64_t t = 0; t * 256 < rows; ++t) {
          const double ci = tc_item_ns(c.kv_dtype, (n.page_count + k - 1) / k, std::min<int64_t>(256, rows - t * 256));
          for (int64_t r = 0; r < k * Hkv; ++r) cost.push_back(ci);
        }
      }
      if (cost.size() == prev_n) continue;  // the chunk caps bind: same split as before
      prev_n = cost.size();
      std::sort(cost.begin(), cost.end(), std::greater<double>());
      const int kc = std::max(1, std::min<int>(K, (int)cost.size()));
      // Loads of the CTAs as a min-heap (negated for std's max-heap).
      load.assign(kc, 0.0);
      double span = 0.0;
      for (double ci : cost) {
        std::pop_heap(load.begin(), load.end());
        load.back() -= ci;
        span = std::max(span, -load.back());
        std::push_heap(load.begin(), load.end());
      }
      const double t = span + merge_bytes / kMergeBytesPerNs;
      if (R == 1 || t < best * 0.98) {
        best = t;
        tc_cap_ns = cap;
      }
    }
  }
  // Pass 1: kernel kind, split-K chunk count and slots of every node.
  p->num_slots = 0;
  for (size_t ni = 0; ni < N; ++ni) {
    const Node& n = p->nodes[ni];
    p->kv_tokens += n.num_tokens;
    const int64_t rows = (int64_t)n.num_q * g;
    const int kind = kind_for(c, p->opts, rows);
    const int rt = row_tile_for(kind);
    p->kv_tokens_by_kind[kind] += n.num_tokens;
    if (kind == kItemTc || kind == kItemTc2) p->tc_row_tokens += rows * n.num_tokens * Hkv;  // all KV heads
    const int64_t row_tiles = (rows + rt - 1) / rt;
    // Split-K chunking. Each extra chunk costs one more partial state per
    // (query, head) written and read back by the merge; allow at most 1/8 of
    // the node's KV bytes for that.
    const double kv_bytes = (double)n.page_count * 2 * Hkv * kPageSize * D * elem;
    const double part_bytes = (double)n.num_q * Hq * (D + 1) * 4.0 * 2.0;
    int64_t kmax = std::max<int64_t>(1, (int64_t)(kv_bytes / (8.0 * part_bytes)));
    int64_t chunk_pages = p->opts.max_chunk_pages > 0 ? p->opts.max_chunk_pages
                          : (row_tiles == 1 ? 16 : (int64_t)1 << 30);
    int64_t k = std::min<int64_t>(kmax, (n.page_count + chunk_pages - 1) / chunk_pages);
    if (kind == kItemTc && tc_sched && p->opts.max_chunk_pages <= 0) {
      // Scheduled tcgen05 items: the chunk count of the chosen time cap.
      k = tc_chunks(c.kv_dtype, n.page_count, std::min<int64_t>(rows, rt), row_tiles * Hkv, tc_cap_ns);
    } else if ((kind == kItemTc || kind == kItemTc2) && p->opts.max_chunk_pages <= 0) {
      // Wide nodes are compute-bound: split their pages so the tensor-core
      // grid covers the SMs (at least 32 pages per chunk), even though each
      // chunk adds a partial state per row (at most 4 chunks, unless fewer
      // than 37 row tiles x KV heads would leave most SMs idle, as for one
      // KV head of a long tree per GPU). A CTA-pair item takes two SMs.
      const int64_t per = row_tiles * Hkv;
      const int64_t units = kind == kItemTc2 ? kPlanSms / 2 : kPlanSms;
      const int64_t target = std::max<int64_t>(1, (units + per / 2) / per);
      // Without the 4-chunk cap, stay within one wave of CTAs.
      const int64_t cap = per * 4 >= kPlanSms ? 4 : std::max<int64_t>(4, units / per);
      k = std::max<int64_t>(k, std::min<int64_t>({target, cap, std::max<int64_t>(1, n.page_count / 32)}));
    }
    k = std::max<int64_t>(1, std::min<int64_t>(k, n.page_count));
    if (n.causal) k = 1;  // items start at the node's first token
    sc.node_k[ni] = (int32_t)k;
    sc.node_kind[ni] = kind;
    // Item size of this node for the longest-first order: pages per chunk x
    // rows per tile.
    sc.keys[ni] = {-((n.page_count + k - 1) / k) * std::min<int64_t>(rows, rt), (int32_t)ni};
    sc.node_slot0[ni] = (int32_t)p->num_slots;
    p->num_slots += k * n.num_q * Hq;
    n_items[kind] += k * Hkv * row_tiles;
    sc.qcount[n.q_begin] += (int32_t)k;
    sc.qcount[n.q_begin + n.num_q] -= (int32_t)k;
  }
  // Each query's path entries in root-to-leaf order (nodes are in DFS
  // pre-order), as CSR: lengths from the difference array, then fill.
  p->path_indptr.assign((size_t)B + 1, 0);
  int32_t run = 0;
  for (int q = 0; q < B; ++q) {
    run += sc.qcount[q];
    p->path_indptr[q + 1] = p->path_indptr[q] + run;
  }
  p->path_slots.resize(p->path_indptr[B]);
  sc.qcursor.assign(p->path_indptr.begin(), p->path_indptr.end() - 1);
  for (int k = 0; k < kNumItemKinds; ++k) p->items[k].resize(n_items[k]);
  int64_t item_fill[kNumItemKinds] = {0, 0, 0, 0, 0};
  // Pass 2: path slots, in DFS order.
  for (size_t ni = 0; ni < N; ++ni) {
    const Node& n = p->nodes[ni];
    for (int32_t ci = 0; ci < sc.node_k[ni]; ++ci) {
      const int32_t slot_base = sc.node_slot0[ni] + ci * n.num_q * Hq;
      for (int32_t qi = 0; qi < n.num_q; ++qi)
        p->path_slots[sc.qcursor[n.q_begin + qi]++] = slot_base + qi * Hq;
    }
  }
  // Pass 3: items, longest first (LPT) so the big shared nodes start early:
  // nodes in decreasing item size (ties in DFS order), each node's items
  // together.
  std::sort(sc.keys.begin(), sc.keys.end());
  for (const auto& key : sc.keys) {
    const size_t ni = (size_t)key.second;
    Node& n = p->nodes[ni];
    const int64_t rows = (int64_t)n.num_q * g;
    const int kind = sc.node_kind[ni];
    const int rt = row_tile_for(kind);
    const int64_t row_tiles = (rows + rt - 1) / rt;
    const int32_t k = sc.node_k[ni];
    n.kind = kind;
    n.k = k;
    n.item_begin = (int32_t)item_fill[kind];
    n.item_count = (int32_t)(k * Hkv * row_tiles);
    WorkItem* out = p->items[kind].data() + item_fill[kind];
    item_fill[kind] += n.item_count;
    for (int32_t ci = 0; ci < k; ++ci) {
      const int32_t pb = (int32_t)((int64_t)ci * n.page_count / k);
      const int32_t pe = (int32_t)((int64_t)(ci + 1) * n.page_count / k);
      const int32_t slot_base = sc.node_slot0[ni] + ci * n.num_q * Hq;
      for (int h = 0; h < Hkv; ++h)
        for (int64_t t = 0; t < row_tiles; ++t) {
          WorkItem it;
          it.page_off = n.page_off + pb;
          it.npages = pe - pb;
          it.last_valid = (pe == n.page_count) ? n.last_valid : kPageSize;
          it.kv_head = h;
          it.row0 = (int32_t)(t * rt);
          it.nrows = (int32_t)std::min<int64_t>(rt, rows - t * rt);
          if (n.causal) {
            // Only the tokens the tile's last query sees.
            const int32_t lim = p->qlimit[n.q_begin + (it.row0 + it.nrows - 1) / g];
            it.npages = (lim + kPageSize - 1) / kPageSize;
            it.last_valid = lim - (it.npages - 1) * kPageSize;
            it.nrows |= kItemCausal;
          }
          if (kind == kItemMma && row_tiles == 1) it.nrows |= kItemSoleReader;
          it.q_begin = n.q_begin;
          it.slot_base = slot_base;
          *out++ = it;
        }
    }
  }
  schedule_tc(p);
  // Deepest node of every DFS query (nodes are in pre-order, so a node's
  // descendants come after it); pages in use.
  p->q_leaf.assign((size_t)B, -1);
  p->live_pages = 0;
  for (size_t ni = 0; ni < N; ++ni) {
    const Node& n = p->nodes[ni];
    p->live_pages += n.page_count;
    for (int32_t q = n.q_begin; q < n.q_begin + n.num_q; ++q) p->q_leaf[q] = (int32_t)ni;
  }
}

static void pack_image(dd_plan* p) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, kAlign);
    return o;
  };
  for (int k = 0; k < kNumItemKinds; ++k)
    p->off_items[k] = take(p->items[k].size() * sizeof(WorkItem));
  p->off_pages = take(p->pages.size() * sizeof(uint32_t));
  p->off_qorder = take(p->query_order.size() * sizeof(int32_t));
  p->off_pindptr = take(p->path_indptr.size() * sizeof(int32_t));
  p->off_pslots = take(p->path_slots.size() * sizeof(int32_t));
  p->off_qlimit = take(p->qlimit.size() * sizeof(int32_t));
  p->off_tc_order = take(p->tc_order.size() * sizeof(int32_t));
  p->off_tc_cta_begin = take(p->tc_cta_begin.size() * sizeof(int32_t));
  // Reused across rebuilds; alignment gaps are never read.
  p->image.resize(std::max<size_t>(off, kAlign));
  auto put = [&](size_t o, const void* src, size_t n) {
    if (n) std::memcpy(p->image.data() + o, src, n);
  };
  for (int k = 0; k < kNumItemKinds; ++k)
    put(p->off_items[k], p->items[k].data(), p->items[k].size() * sizeof(WorkItem));
  put(p->off_pages, p->pages.data(), p->pages.size() * 4);
  put(p->off_qorder, p->query_order.data(), p->query_order.size() * 4);
  put(p->off_pindptr, p->path_indptr.data(), p->path_indptr.size() * 4);
  put(p->off_pslots, p->path_slots.data(), p->path_slots.size() * 4);
  put(p->off_qlimit, p->qlimit.data(), p->qlimit.size() * 4);
  put(p->off_tc_order, p->tc_order.data(), p->tc_order.size() * 4);
  put(p->off_tc_cta_begin, p->tc_cta_begin.data(), p->tc_cta_begin.size() * 4);
}

}  // namespace dd

dd_plan::~dd_plan() {
  dd::release_staging(this);
  delete scratch;
}

using namespace dd;

extern "C" {

const char* dd_version(void) { return "dendrite_b200 0.1.0 (sm_100a)"; }

const char* dd_last_error(void) { return g_last_error.c_str(); }

int dd_validate_config(const dd_attn_config* cfg) { return check_config(cfg); }

int dd_plan_create(const dd_attn_config* cfg, int32_t batch_size, const int32_t* block_indptr,
                   const uint32_t* block_ids, const int32_t* num_tokens,
                   const dd_plan_options* opts, dd_plan** out_plan) {
  if (!out_plan) return fail(DD_ERR_INVALID_ARGUMENT, "out_plan is NULL");
  *out_plan = nullptr;
  int st = check_config(cfg);
  if (st) return st;
  if (batch_size < 0) return fail(DD_ERR_INVALID_ARGUMENT, "batch_size must be >= 0");
  if (batch_size > 0 && (!block_indptr || !num_tokens))
    return fail(DD_ERR_INVALID_ARGUMENT, "block_indptr / num_tokens is NULL");
  if (batch_size > 0 && block_indptr[batch_size] > 0 && !block_ids)
    return fail(DD_ERR_INVALID_ARGUMENT, "block_ids is NULL");
  dd_plan* p = new (std::nothrow) dd_plan();
  if (!p) return fail(DD_ERR_ALLOCATION, "host allocation failed");
  p->cfg = *cfg;
  if (p->cfg.scale <= 0.f) p->cfg.scale = 1.0f / std::sqrt((float)cfg->head_dim);
  if (opts) {
    p->opts = *opts;
  } else {
    p->opts = dd_plan_options{1, 0, 1, 0, 0};
  }
  p->batch_size = batch_size;
  try {
    reset_plan(p);
    st = build_nodes(p, block_indptr, block_ids, num_tokens);
    if (st) {
      delete p;
      return st;
    }
    build_items(p);
    if (p->num_slots > INT32_MAX) {
      delete p;
      return fail(DD_ERR_INVALID_ARGUMENT, "plan too large (partial slots exceed 2^31)");
    }
    pack_image(p);
  } catch (const std::bad_alloc&) {
    delete p;
    return fail(DD_ERR_ALLOCATION, "host allocation failed while planning");
  }
  *out_plan = p;
  return DD_OK;
}

int dd_plan_rebuild(dd_plan* p, int32_t batch_size, const int32_t* block_indptr,
                    const uint32_t* block_ids, const int32_t* num_tokens) {
  if (!p) return fail(DD_ERR_INVALID_ARGUMENT, "plan is NULL");
  if (batch_size < 0) return fail(DD_ERR_INVALID_ARGUMENT, "batch_size must be >= 0");
  if (batch_size > 0 && (!block_indptr || !num_tokens))
    return fail(DD_ERR_INVALID_ARGUMENT, "block_indptr / num_tokens is NULL");
  if (batch_size > 0 && block_indptr[batch_size] > 0 && !block_ids)
    return fail(DD_ERR_INVALID_ARGUMENT, "block_ids is NULL");
  p->batch_size = batch_size;
  try {
    reset_plan(p);
    int st = build_nodes(p, block_indptr, block_ids, num_tokens);
    if (!st) {
      build_items(p);
      if (p->num_slots > INT32_MAX) st = fail(DD_ERR_INVALID_ARGUMENT, "plan too large (partial slots exceed 2^31)");
    }
    if (!st) pack_image(p);
    if (st) {
      reset_plan(p);  // leave an empty, valid plan behind
      p->batch_size = 0;
      pack_image(p);
    }
    return st;
  } catch (const std::bad_alloc&) {
    reset_plan(p);
    p->batch_size = 0;
    return fail(DD_ERR_ALLOCATION, "host allocation failed while planning");
  }
}

// Causal prefill plan. Sequence s holds prefix_len[s] + num_new[s] tokens;
// its new tokens are queries (numbered sequence-major) and new token i sees
// tokens [0, prefix_len[s] + i]. The full pages of the prefixes form a radix
// tree (shared prefix pages are read once for all the new tokens below them,
// with no mask); below it, each sequence has a causal node that starts at
// the page holding token prefix_len[s] (so a partial prefix page is part of
// it) and whose query i sees its first prefix_len[s] % 16 + i + 1 tokens.
int dd_plan_create_prefill(const dd_attn_config* cfg, int32_t num_seqs, const int32_t* block_indptr,
                           const uint32_t* block_ids, const int32_t* prefix_len,
                           const int32_t* num_new, const dd_plan_options* opts,
                           dd_plan** out_plan) {
  if (!out_plan) return fail(DD_ERR_INVALID_ARGUMENT, "out_plan is NULL");
  *out_plan = nullptr;
  int st = check_config(cfg);
  if (st) return st;
  if (num_seqs < 0) return fail(DD_ERR_INVALID_ARGUMENT, "num_seqs must be >= 0");
  if (num_seqs > 0 && (!block_indptr || !prefix_len || !num_new))
    return fail(DD_ERR_INVALID_ARGUMENT, "block_indptr / prefix_len / num_new is NULL");
  if (num_seqs > 0 && block_indptr[num_seqs] > 0 && !block_ids)
    return fail(DD_ERR_INVALID_ARGUMENT, "block_ids is NULL");
  int64_t total = 0;
  for (int s = 0; s < num_seqs; ++s) {
    const int64_t nb = (int64_t)block_indptr[s + 1] - block_indptr[s];
    if (nb < 0) return fail(DD_ERR_INVALID_ARGUMENT, "block_indptr must be non-decreasing");
    if (prefix_len[s] < 0 || num_new[s] < 0) return fail(DD_ERR_INVALID_ARGUMENT, "prefix_len / num_new must be >= 0");
    if ((int64_t)prefix_len[s] + num_new[s] > nb * kPageSize)
      return fail(DD_ERR_INVALID_ARGUMENT, "prefix_len + num_new of sequence " + std::to_string(s) +
                                               " exceeds its block table");
    total += num_new[s];
  }
  if (total > INT32_MAX) return fail(DD_ERR_INVALID_ARGUMENT, "too many prefill tokens");
  dd_plan* p = new (std::nothrow) dd_plan();
  if (!p) return fail(DD_ERR_ALLOCATION, "host allocation failed");
  p->cfg = *cfg;
  if (p->cfg.scale <= 0.f) p->cfg.scale = 1.0f / std::sqrt((float)cfg->head_dim);
  p->opts = opts ? *opts : dd_plan_options{1, 0, 1, 0, 0};
  p->opts.cta_pairs = 0;  // the CTA-pair kernel has no causal mask
  try {
    reset_plan(p);
    // 1. Radix tree over the sequences' full prefix pages (queries =
    //    sequences for now).
    std::vector<int32_t> full((size_t)num_seqs);
    for (int s = 0; s < num_seqs; ++s) full[s] = (prefix_len[s] / kPageSize) * kPageSize;
    p->batch_size = num_seqs;
    st = build_nodes(p, block_indptr, block_ids, full.data());
    if (st) {
      delete p;
      return st;
    }
    // 2. Re-number queries: sequence at DFS position d owns new-token
    //    queries [qd[d], qd[d + 1]).
    const std::vector<int32_t> seq_order = p->query_order;
    std::vector<int32_t> qd((size_t)num_seqs + 1, 0), base((size_t)num_seqs + 1, 0);
    for (int d = 0; d < num_seqs; ++d) qd[d + 1] = qd[d] + num_new[seq_order[d]];
    for (int s = 0; s < num_seqs; ++s) base[s + 1] = base[s] + num_new[s];
    std::vector<int32_t> deepest((size_t)num_seqs, -1);
    for (size_t ni = 0; ni < p->nodes.size(); ++ni) {
      Node& n = p->nodes[ni];
      for (int32_t d = n.q_begin; d < n.q_begin + n.num_q; ++d) deepest[d] = (int32_t)ni;
      const int32_t b0 = qd[n.q_begin], b1 = qd[n.q_begin + n.num_q];
      n.q_begin = b0;
      n.num_q = b1 - b0;
    }
    p->batch_size = (int32_t)total;
    p->causal = true;
    p->query_order.assign((size_t)total, 0);
    p->qlimit.assign((size_t)total, 0);
    p->kv_tokens_flat = 0;
    // 3. One causal node per sequence with new tokens.
    for (int d = 0; d < num_seqs; ++d) {
      const int s = seq_order[d];
      const int32_t n_new = num_new[s], pre = prefix_len[s];
      for (int32_t i = 0; i < n_new; ++i) {
        p->query_order[qd[d] + i] = base[s] + i;
        p->qlimit[qd[d] + i] = pre % kPageSize + i + 1;
      }
      p->kv_tokens_flat += (int64_t)n_new * pre + (int64_t)n_new * (n_new + 1) / 2;
      if (n_new == 0) continue;
      const int32_t first = pre / kPageSize, end = (pre + n_new + kPageSize - 1) / kPageSize;
      const uint32_t* ids = block_ids + block_indptr[s];
      for (int32_t i = first; i < end; ++i)
        if (ids[i] >= (uint32_t)cfg->num_pages) {
          delete p;
          return fail(DD_ERR_INVALID_ARGUMENT, "invalid block id: " + std::to_string(ids[i]));
        }
      Node n;
      n.parent = deepest[d];
      n.depth = n.parent < 0 ? 0 : p->nodes[n.parent].depth + 1;
      n.q_begin = qd[d];
      n.num_q = n_new;
      n.num_tokens = pre % kPageSize + n_new;
      n.page_off = (int32_t)p->pages.size();
      n.page_count = end - first;
      n.last_valid = pre + n_new - (end - 1) * kPageSize;
      n.causal = true;
      p->pages.insert(p->pages.end(), ids + first, ids + end);
      p->nodes.push_back(n);
      p->max_depth = std::max(p->max_depth, n.depth + 1);
    }
    build_items(p);
    if (p->num_slots > INT32_MAX) {
      delete p;
      return fail(DD_ERR_INVALID_ARGUMENT, "plan too large (partial slots exceed 2^31)");
    }
    pack_image(p);
  } catch (const std::bad_alloc&) {
    delete p;
    return fail(DD_ERR_ALLOCATION, "host allocation failed while planning");
  }
  *out_plan = p;
  return DD_OK;
}

// One decode step in place: query b (in the batch's order) gained
// tokens_added[b] (0 or 1) tokens; a token that starts a new block went to
// block new_block[b]. Only a query whose deepest node is its own (no other
// query shares its last pages) can grow in place: its node gains the token
// (and the block), and the node's items are re-cut. Any other change returns
// DD_ERR_NOT_AVAILABLE with the plan unchanged; the caller re-plans with
// dd_plan_rebuild from the full tables.
int dd_plan_advance(dd_plan* p, const int32_t* tokens_added, const uint32_t* new_block) {
  if (!p || !tokens_added) return fail(DD_ERR_INVALID_ARGUMENT, "plan / tokens_added is NULL");
  if (p->causal) return fail(DD_ERR_NOT_AVAILABLE, "prefill plans are not advanced; re-plan");
  if (!p->opts.share_prefixes) return fail(DD_ERR_NOT_AVAILABLE, "flat plans are not advanced; re-plan");
  const int B = p->batch_size;
  PlanScratch& sc = *p->scratch;
  std::vector<int32_t>& pos = sc.qcursor;  // DFS position of each query
  pos.assign((size_t)B, 0);
  for (int d = 0; d < B; ++d) pos[p->query_order[d]] = d;
  int64_t grow_pages = 0;
  for (int b = 0; b < B; ++b) {
    const int32_t t = tokens_added[b];
    if (t == 0) continue;
    if (t != 1) return fail(DD_ERR_INVALID_ARGUMENT, "tokens_added must be 0 or 1");
    const int32_t leaf = p->q_leaf[pos[b]];
    if (leaf < 0 || p->nodes[leaf].num_q != 1)
      return fail(DD_ERR_NOT_AVAILABLE, "query " + std::to_string(b) + " shares its last pages; re-plan");
    if (p->nodes[leaf].last_valid == kPageSize) {
      if (!new_block) return fail(DD_ERR_INVALID_ARGUMENT, "new_block is NULL");
      if (new_block[b] >= (uint32_t)p->cfg.num_pages)
        return fail(DD_ERR_INVALID_ARGUMENT, "invalid block id: " + std::to_string(new_block[b]));
      grow_pages += p->nodes[leaf].page_count + 1;
    }
  }
  // Moved runs leave dead entries behind; past as many dead as live ids,
  // re-plan (which compacts).
  if ((int64_t)p->pages.size() + grow_pages > 2 * (p->live_pages + grow_pages) + 1024)
    return fail(DD_ERR_NOT_AVAILABLE, "page list needs compaction; re-plan");
  const int Hkv = p->cfg.num_kv_heads, g = p->cfg.num_qo_heads / Hkv;
  for (int b = 0; b < B; ++b) {
    if (tokens_added[b] == 0) continue;
    Node& n = p->nodes[p->q_leaf[pos[b]]];
    if (n.last_valid == kPageSize) {
      // The node's run moves to the end of the page list, followed by the new block.
      if ((size_t)(n.page_off + n.page_count) != p->pages.size()) {
        const size_t off = p->pages.size();
        p->pages.resize(off + n.page_count);
        std::memcpy(p->pages.data() + off, p->pages.data() + n.page_off, (size_t)n.page_count * 4);
        n.page_off = (int32_t)off;
      }
      p->pages.push_back(new_block[b]);
      ++n.page_count;
      ++p->live_pages;
      n.last_valid = 1;
    } else {
      ++n.last_valid;
    }
    ++n.num_tokens;
    ++p->kv_tokens;
    ++p->kv_tokens_flat;
    p->kv_tokens_by_kind[n.kind] += 1;
    // Re-cut the node's items: [chunk][KV head][row tile], as the builder emits them.
    const int rt = row_tile_for(n.kind);
    const int32_t row_tiles = (int32_t)((n.num_q * g + rt - 1) / rt);
    WorkItem* it = p->items[n.kind].data() + n.item_begin;
    for (int32_t ci = 0; ci < n.k; ++ci) {
      const int32_t pb = (int32_t)((int64_t)ci * n.page_count / n.k);
      const int32_t pe = (int32_t)((int64_t)(ci + 1) * n.page_count / n.k);
      for (int32_t j = 0; j < Hkv * row_tiles; ++j, ++it) {
        it->page_off = n.page_off + pb;
        it->npages = pe - pb;
        it->last_valid = pe == n.page_count ? n.last_valid : kPageSize;
      }
    }
  }
  pack_image(p);
  // The image's layout changed: a decode before the next dd_plan_upload must
  // fail instead of reading the old image at the new offsets.
  p->device_base = nullptr;
  p->device_id = -1;
  return DD_OK;
}

void dd_plan_destroy(dd_plan* plan) { delete plan; }

int dd_plan_get_info(const dd_plan* p, dd_plan_info* info) {
  if (!p || !info) return fail(DD_ERR_INVALID_ARGUMENT, "NULL argument");
  info->batch_size = p->batch_size;
  info->num_nodes = (int32_t)p->nodes.size();
  int32_t n = 0;
  for (auto& v : p->items) n += (int32_t)v.size();
  info->num_items = n;
  info->max_depth = p->max_depth;
  info->kv_tokens = p->kv_tokens;
  info->kv_tokens_flat = p->kv_tokens_flat;
  for (int k = 0; k < kNumItemKinds; ++k) info->kv_tokens_by_kernel[k] = p->kv_tokens_by_kind[k];
  info->tc_row_tokens = p->tc_row_tokens;
  info->tc_ctas = p->tc_ctas > 0 ? p->tc_ctas : (int32_t)p->items[kItemTc].size();
  info->workspace_bytes = plan_workspace_bytes(p);
  info->device_bytes = p->image.size();
  return DD_OK;
}

int dd_plan_export_nodes(const dd_plan* p, int32_t* parent, int32_t* q_begin, int32_t* num_q,
                         int32_t* num_tokens, int32_t* page_offset, int32_t* page_count,
                         uint32_t* pages, int32_t* query_order) {
  if (!p) return fail(DD_ERR_INVALID_ARGUMENT, "plan is NULL");
  // Pages are exported node after node (offsets into that list), without
  // the dead runs dd_plan_advance leaves in the plan's own list.
  int32_t off = 0;
  for (size_t i = 0; i < p->nodes.size(); ++i) {
    const Node& n = p->nodes[i];
    if (parent) parent[i] = n.parent;
    if (q_begin) q_begin[i] = n.q_begin;
    if (num_q) num_q[i] = n.num_q;
    if (num_tokens) num_tokens[i] = n.num_tokens;
    if (page_offset) page_offset[i] = off;
    if (page_count) page_count[i] = n.page_count;
    if (pages && n.page_count)
      std::memcpy(pages + off, p->pages.data() + n.page_off, (size_t)n.page_count * 4);
    off += n.page_count;
  }
  if (query_order && !p->query_order.empty())
    std::memcpy(query_order, p->query_order.data(), p->query_order.size() * 4);
  return DD_OK;
}

}  // extern "C"
