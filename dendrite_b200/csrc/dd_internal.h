// Internal structures shared by the host planner (planner.cpp) and the CUDA
// kernels. Not part of the public C ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/dendrite_b200.h"

namespace dd {

constexpr int kPageSize = 16;           // tokens per page (cache/mod.rs:61)
constexpr size_t kWsHeaderBytes = 256;  // workspace header: device error words
constexpr size_t kAlign = 256;

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Kernel families a work item can be routed to.
enum ItemKind : int32_t {
  kItemSimple = 0,  // CUDA-core kernel (any dtype, any head_dim) — f32 KV path
  kItemMma = 1,     // warp-level tensor-core tiles, <= 64 query rows per item
  kItemTc = 2,      // tcgen05 (TMEM accumulators), up to 256 query rows per item
  kItemTc2 = 3,     // tcgen05 on a CTA pair (cta_group::2), up to 512 rows per item
  kItemReserved = 4,  // unused (keeps the ABI's per-kernel token array at 5 entries)
  kNumItemKinds = 5
};

// One unit of kernel work: rows [row0, row0 + nrows) of a plan node for one
// KV head, over the node's pages [page_off, page_off + npages) of the plan's
// flat page list. Row r of a node stands for query (q_begin + r / g) in DFS
// order and its (r % g)-th query head of this KV head.
struct WorkItem {
  int32_t page_off;    // into the plan's flat page-id array
  int32_t npages;
  int32_t last_valid;  // valid tokens in the last page of this item (1..16)
  int32_t kv_head;
  int32_t row0;
  int32_t nrows;
  int32_t q_begin;     // DFS position of the node's first query
  int32_t slot_base;   // partial-state slot of (node, chunk, query 0, head 0)
};
static_assert(sizeof(WorkItem) == 32, "WorkItem layout");
// Item flags in the high bits of nrows (kernels mask with kItemRowsMask):
//  - kItemSoleReader (streaming items): the only reader of its pages in the
//    launch (its node has one row tile); streams them L2 evict-first;
//  - kItemCausal (prefill plans): the item's node is a causal suffix; its row
//    for DFS query p sees the node's first qlimit[p] tokens.
constexpr int32_t kItemSoleReader = 1 << 16;
constexpr int32_t kItemCausal = 1 << 17;
constexpr int32_t kItemRowsMask = 0xffff;

// Device-side view of an uploaded plan (pointers into the caller's buffer).
struct DevicePlan {
  const WorkItem* items[kNumItemKinds];
  int32_t num_items[kNumItemKinds];
  const uint32_t* pages;       // flat page ids of all nodes
  const int32_t* query_order;  // DFS position -> query index
  const int32_t* path_indptr;  // [batch+1] per DFS position
  const int32_t* path_slots;   // slot of (node, chunk, this query, head 0)
};

struct Node {
  int32_t parent = -1;
  int32_t q_begin = 0;
  int32_t num_q = 0;
  int32_t num_tokens = 0;
  int32_t page_off = 0;
  int32_t page_count = 0;
  int32_t last_valid = kPageSize;
  int32_t depth = 0;
  bool causal = false;  // prefill suffix: query p sees its first qlimit[p] tokens
  // Set by the item builder: kernel kind, split-K chunks, and the node's
  // items [item_begin, item_begin + item_count) of items[kind].
  int32_t kind = 0, k = 1, item_begin = 0, item_count = 0;
};

}  // namespace dd

namespace dd {
struct PlanScratch;  // planner.cpp: working buffers kept across dd_plan_rebuild
}

// The opaque plan handed across the C ABI.
struct dd_plan {
  dd_attn_config cfg;
  dd_plan_options opts;
  int32_t batch_size = 0;
  std::vector<dd::Node> nodes;
  std::vector<uint32_t> pages;
  std::vector<int32_t> query_order;
  std::vector<int32_t> path_indptr;
  std::vector<int32_t> path_slots;
  std::vector<dd::WorkItem> items[dd::kNumItemKinds];
  int64_t num_slots = 0;
  int64_t kv_tokens = 0;
  int64_t kv_tokens_flat = 0;
  int64_t kv_tokens_by_kind[dd::kNumItemKinds] = {0, 0, 0, 0, 0};
  int64_t tc_row_tokens = 0;
  int32_t max_depth = 0;
  // Causal (prefill) plans: tokens of its node visible to each DFS query;
  // items then cover their node from its first token and are not split.
  bool causal = false;
  std::vector<int32_t> qlimit;
  size_t off_qlimit = 0;
  // Deepest node of each DFS query (-1: empty table), for dd_plan_advance.
  std::vector<int32_t> q_leaf;
  int64_t live_pages = 0;  // pages referenced by nodes (the rest of `pages` is dead)
  // Packed host image of everything the device needs, and its layout.
  std::vector<uint8_t> image;
  size_t off_items[dd::kNumItemKinds] = {0, 0, 0, 0, 0};
  size_t off_pages = 0, off_qorder = 0, off_pindptr = 0, off_pslots = 0;
  // Schedule of the tcgen05 items onto tc_ctas CTAs: CTA c runs items
  // tc_order[tc_cta_begin[c] .. tc_cta_begin[c + 1]).
  int32_t tc_ctas = 0;
  std::vector<int32_t> tc_order, tc_cta_begin;
  size_t off_tc_order = 0, off_tc_cta_begin = 0;
  // Set by dd_plan_upload.
  const void* device_base = nullptr;
  int device_id = -1;
  // Pinned host copy of the image for dd_plan_upload (api.cu), so the upload
  // is a true asynchronous copy, and the event of its last copy.
  void* staging = nullptr;
  size_t staging_bytes = 0;
  void* staging_event = nullptr;
  int staging_device = -1;
  dd::PlanScratch* scratch = nullptr;
  ~dd_plan();
};

namespace dd {
// Frees the plan's pinned upload staging (api.cu).
void release_staging(dd_plan* p);
// Thread-local error message used by dd_last_error().
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_config(const dd_attn_config* cfg);
size_t plan_workspace_bytes(const dd_plan* p);
}  // namespace dd
