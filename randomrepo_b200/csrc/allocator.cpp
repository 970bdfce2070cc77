// Host block allocator of the paged-KV pool (C ABI in include/pkv_b200.h).
//
// Semantics follow AgentRL's PagedKVAllocator (agentrl/generation/paged_kv.py:25-175):
//  * allocation always takes the lowest free block id -- the reference pops a
//    min-heap (paged_kv.py:42-43,162), so its order is exactly "smallest free
//    id"; here a two-level bitmap answers that in O(total/4096) words;
//  * a block counts as reused when an id that was handed out before is handed
//    out again (paged_kv.py:163-166);
//  * the high watermark is updated after successful reserve/append only
//    (paged_kv.py:90,109);
//  * failure paths keep the reference's partial effects: a reserve that runs
//    out part-way leaves the ids it already took out of the free set (they are
//    owned by no sequence), an append that runs out keeps the blocks it already
//    appended and leaves the token count unchanged.
// Extension with no reference counterpart: per-block refcounts, fork (a child
// shares its parent's blocks) and copy-on-write of a shared partial tail block
// on the first append after a fork.  Without forks every refcount is 1 and all
// results equal the reference's.
//
// Every call also records which device-mirror entries changed (block-table
// entries, refcounts, context lengths) and which block copies copy-on-write
// needs, so the device tables can be brought up to date with one upload and
// one kernel (pkv_apply_updates).

#include "pkv_b200.h"

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <queue>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "pkv_error.h"

namespace {

struct Sequence {
  int32_t row = -1;
  int64_t tokens = 0;
  std::vector<int32_t> blocks;
};

}  // namespace

struct pkv_allocator {
  int64_t total = 0;
  int64_t block_size = 0;

  // Free-set bitmap (bit = 1 means free) with a summary word per 64 words.
  std::vector<uint64_t> words;
  std::vector<uint64_t> summary;
  int64_t free_count = 0;

  std::vector<uint8_t> touched;
  int64_t reuse = 0;
  int64_t high = 0;

  std::vector<int32_t> refcount;
  int64_t shared = 0;

  std::unordered_map<int64_t, Sequence> seqs;
  std::vector<Sequence*> row_owner;
  // Bumped whenever a sequence is created or destroyed; a decode step over
  // the same ids as the previous one reuses that step's id -> sequence lookup.
  uint64_t generation = 0;
  std::vector<int64_t> step_ids;
  std::vector<Sequence*> step_seqs;
  uint64_t step_generation = ~0ull;
  std::priority_queue<int32_t, std::vector<int32_t>, std::greater<int32_t>> free_rows;
  int64_t max_cols = 0;

  // Device-mirror change record.
  std::unordered_set<uint64_t> dirty_table;
  std::vector<uint8_t> ref_dirty;
  std::vector<int32_t> ref_dirty_list;
  std::vector<uint8_t> len_dirty;
  std::vector<int32_t> len_dirty_list;
  std::vector<std::pair<int32_t, int32_t>> copies;

  void set_free(int64_t b) {
    words[b >> 6] |= (1ull << (b & 63));
    summary[b >> 12] |= (1ull << ((b >> 6) & 63));
    ++free_count;
  }

  // Lowest free id, or -1.
  int64_t take_lowest() {
    for (size_t s = 0; s < summary.size(); ++s) {
      uint64_t sw = summary[s];
      if (!sw) continue;
      int64_t w = (int64_t)(s << 6) + __builtin_ctzll(sw);
      uint64_t word = words[w];
      int64_t b = (w << 6) + __builtin_ctzll(word);
      word &= word - 1;
      words[w] = word;
      if (!word) summary[s] &= ~(1ull << (w & 63));
      --free_count;
      return b;
    }
    return -1;
  }

  bool allocate(int32_t* out) {
    int64_t b = take_lowest();
    if (b < 0) {
      pkv_set_error("PagedKVAllocator ran out of free blocks.");
      return false;
    }
    if (touched[b]) {
      ++reuse;
    } else {
      touched[b] = 1;
    }
    *out = (int32_t)b;
    return true;
  }

  void set_ref(int32_t b, int32_t v) {
    int32_t old = refcount[b];
    if (old > 1 && v <= 1) --shared;
    if (old <= 1 && v > 1) ++shared;
    refcount[b] = v;
    if (!ref_dirty[b]) {
      ref_dirty[b] = 1;
      ref_dirty_list.push_back(b);
    }
  }

  void mark_entry(int32_t row, int64_t col) {
    dirty_table.insert(((uint64_t)(uint32_t)row << 32) | (uint64_t)(uint32_t)col);
  }

  void mark_len(int32_t row) {
    if ((size_t)row >= len_dirty.size()) len_dirty.resize(row + 1, 0);
    if (!len_dirty[row]) {
      len_dirty[row] = 1;
      len_dirty_list.push_back(row);
    }
  }

  int32_t take_row(Sequence* s) {
    int32_t r;
    if (!free_rows.empty()) {
      r = free_rows.top();
      free_rows.pop();
    } else {
      r = (int32_t)row_owner.size();
      row_owner.push_back(nullptr);
    }
    row_owner[r] = s;
    return r;
  }

  int64_t required(int64_t tokens) const { return tokens == 0 ? 0 : (tokens + block_size - 1) / block_size; }

  void update_high() { high = std::max(high, total - free_count); }

  void note_cols(size_t n) { max_cols = std::max<int64_t>(max_cols, (int64_t)n); }

  // append_tokens body; `track` = record growth entries and the length as dirty.
  int32_t append(Sequence& s, int64_t count, bool track, int32_t* new_block) {
    if (new_block) *new_block = -1;
    if (count == 0) return PKV_OK;
    if (!s.blocks.empty() && s.tokens % block_size != 0 && refcount[s.blocks.back()] > 1) {
      int32_t src = s.blocks.back(), dst;
      if (!allocate(&dst)) return PKV_ERR_RUNTIME;
      set_ref(src, refcount[src] - 1);
      set_ref(dst, 1);
      s.blocks.back() = dst;
      copies.emplace_back(src, dst);
      mark_entry(s.row, (int64_t)s.blocks.size() - 1);
    }
    int64_t total_tokens = s.tokens + count;
    int64_t need = required(total_tokens);
    while ((int64_t)s.blocks.size() < need) {
      int32_t b;
      if (!allocate(&b)) return PKV_ERR_RUNTIME;
      set_ref(b, 1);
      s.blocks.push_back(b);
      note_cols(s.blocks.size());
      if (track) {
        mark_entry(s.row, (int64_t)s.blocks.size() - 1);
      } else if (new_block) {
        *new_block = b;
      }
    }
    s.tokens = total_tokens;
    if (track) mark_len(s.row);
    update_high();
    return PKV_OK;
  }
};

extern "C" {

pkv_allocator* pkv_allocator_create(int64_t total_blocks, int64_t block_size_tokens, int32_t* status) {
  pkv_clear_error();
  if (total_blocks <= 0) {
    pkv_set_error("total_blocks must be > 0.");
    if (status) *status = PKV_ERR_VALUE;
    return nullptr;
  }
  if (block_size_tokens <= 0) {
    pkv_set_error("block_size_tokens must be > 0.");
    if (status) *status = PKV_ERR_VALUE;
    return nullptr;
  }
  if (total_blocks > INT32_MAX) {
    pkv_set_error("total_blocks must fit in int32 (device block ids are int32).");
    if (status) *status = PKV_ERR_VALUE;
    return nullptr;
  }
  auto* a = new pkv_allocator();
  a->total = total_blocks;
  a->block_size = block_size_tokens;
  a->words.assign((total_blocks + 63) / 64, 0);
  a->summary.assign((a->words.size() + 63) / 64, 0);
  for (int64_t b = 0; b < total_blocks; ++b) a->set_free(b);
  a->touched.assign(total_blocks, 0);
  a->refcount.assign(total_blocks, 0);
  a->ref_dirty.assign(total_blocks, 0);
  if (status) *status = PKV_OK;
  return a;
}

void pkv_allocator_destroy(pkv_allocator* a) { delete a; }

int32_t pkv_allocator_reserve(pkv_allocator* a, int64_t sequence_id, int64_t token_count) {
  pkv_clear_error();
  if (a->seqs.count(sequence_id)) {
    pkv_set_error("sequence_id " + std::to_string(sequence_id) + " is already allocated.");
    return PKV_ERR_VALUE;
  }
  if (token_count < 0) {
    pkv_set_error("token_count must be >= 0.");
    return PKV_ERR_VALUE;
  }
  int64_t need = a->required(token_count);
  std::vector<int32_t> blocks;
  blocks.reserve(need);
  for (int64_t i = 0; i < need; ++i) {
    int32_t b;
    if (!a->allocate(&b)) {
      // The reference's list comprehension has already popped these ids; they
      // stay out of the free set, belong to no sequence and keep refcount 0.
      return PKV_ERR_RUNTIME;
    }
    blocks.push_back(b);
  }
  Sequence& s = a->seqs[sequence_id];
  ++a->generation;
  s.tokens = token_count;
  s.blocks = std::move(blocks);
  s.row = a->take_row(&s);
  for (size_t j = 0; j < s.blocks.size(); ++j) {
    a->set_ref(s.blocks[j], 1);
    a->mark_entry(s.row, (int64_t)j);
  }
  a->note_cols(s.blocks.size());
  a->mark_len(s.row);
  a->update_high();
  return PKV_OK;
}

int32_t pkv_allocator_append_tokens(pkv_allocator* a, int64_t sequence_id, int64_t token_count) {
  pkv_clear_error();
  if (token_count < 0) {
    pkv_set_error("token_count must be >= 0.");
    return PKV_ERR_VALUE;
  }
  auto it = a->seqs.find(sequence_id);
  if (it == a->seqs.end()) {
    pkv_set_error("Unknown sequence_id " + std::to_string(sequence_id) + ".");
    return PKV_ERR_KEY;
  }
  return a->append(it->second, token_count, /*track=*/true, nullptr);
}

int32_t pkv_allocator_release(pkv_allocator* a, int64_t sequence_id) {
  pkv_clear_error();
  auto it = a->seqs.find(sequence_id);
  if (it == a->seqs.end()) {
    pkv_set_error("Unknown sequence_id " + std::to_string(sequence_id) + ".");
    return PKV_ERR_KEY;
  }
  Sequence& s = it->second;
  for (int32_t b : s.blocks) {
    a->set_ref(b, a->refcount[b] - 1);
    if (a->refcount[b] == 0) a->set_free(b);
  }
  a->row_owner[s.row] = nullptr;
  a->free_rows.push(s.row);
  a->mark_len(s.row);
  a->seqs.erase(it);
  ++a->generation;
  return PKV_OK;
}

int32_t pkv_allocator_fork(pkv_allocator* a, int64_t parent_id, int64_t child_id) {
  pkv_clear_error();
  if (a->seqs.count(child_id)) {
    pkv_set_error("sequence_id " + std::to_string(child_id) + " is already allocated.");
    return PKV_ERR_VALUE;
  }
  auto it = a->seqs.find(parent_id);
  if (it == a->seqs.end()) {
    pkv_set_error("Unknown sequence_id " + std::to_string(parent_id) + ".");
    return PKV_ERR_KEY;
  }
  std::vector<int32_t> blocks = it->second.blocks;
  int64_t tokens = it->second.tokens;
  Sequence& c = a->seqs[child_id];  // may rehash; `it` is not used after this
  ++a->generation;
  c.tokens = tokens;
  c.blocks = std::move(blocks);
  c.row = a->take_row(&c);
  for (size_t j = 0; j < c.blocks.size(); ++j) {
    a->set_ref(c.blocks[j], a->refcount[c.blocks[j]] + 1);
    a->mark_entry(c.row, (int64_t)j);
  }
  a->mark_len(c.row);
  return PKV_OK;
}

int32_t pkv_allocator_logical_to_physical(pkv_allocator* a, int64_t sequence_id, int64_t logical_block_index,
                                          int64_t* block_out) {
  pkv_clear_error();
  if (logical_block_index < 0) {
    pkv_set_error("logical_block_index must be >= 0.");
    return PKV_ERR_VALUE;
  }
  auto it = a->seqs.find(sequence_id);
  if (it == a->seqs.end()) {
    // The reference indexes its dict directly: KeyError(sequence_id).
    pkv_set_error(std::to_string(sequence_id));
    return PKV_ERR_KEY;
  }
  if (logical_block_index >= (int64_t)it->second.blocks.size()) {
    pkv_set_error("list index out of range");
    return PKV_ERR_INDEX;
  }
  *block_out = it->second.blocks[logical_block_index];
  return PKV_OK;
}

int32_t pkv_allocator_view(pkv_allocator* a, int64_t sequence_id, int64_t* token_count, int32_t* blocks,
                           int64_t capacity, int64_t* num_blocks) {
  pkv_clear_error();
  auto it = a->seqs.find(sequence_id);
  if (it == a->seqs.end()) {
    pkv_set_error("Unknown sequence_id " + std::to_string(sequence_id) + ".");
    return PKV_ERR_KEY;
  }
  const Sequence& s = it->second;
  if (token_count) *token_count = s.tokens;
  if (num_blocks) *num_blocks = (int64_t)s.blocks.size();
  if (blocks) {
    int64_t n = std::min<int64_t>(capacity, (int64_t)s.blocks.size());
    std::memcpy(blocks, s.blocks.data(), sizeof(int32_t) * n);
  }
  return PKV_OK;
}

int32_t pkv_allocator_has_sequence(pkv_allocator* a, int64_t sequence_id) {
  return a->seqs.count(sequence_id) ? 1 : 0;
}

int32_t pkv_allocator_get_stats(pkv_allocator* a, pkv_allocator_stats* out) {
  out->total_blocks = a->total;
  out->block_size_tokens = a->block_size;
  out->free_block_count = a->free_count;
  out->used_block_count = a->total - a->free_count;
  out->block_reuse_count = a->reuse;
  out->max_blocks_in_use = a->high;
  out->resident_sequence_count = (int64_t)a->seqs.size();
  out->row_capacity = (int64_t)a->row_owner.size();
  out->max_blocks_per_row = a->max_cols;
  out->shared_block_count = a->shared;
  return PKV_OK;
}

int32_t pkv_allocator_refcount(pkv_allocator* a, int64_t block, int32_t* out) {
  pkv_clear_error();
  if (block < 0 || block >= a->total) {
    pkv_set_error("block id out of range");
    return PKV_ERR_INDEX;
  }
  *out = a->refcount[block];
  return PKV_OK;
}

int32_t pkv_allocator_row(pkv_allocator* a, int64_t sequence_id, int32_t* row_out) {
  pkv_clear_error();
  auto it = a->seqs.find(sequence_id);
  if (it == a->seqs.end()) {
    pkv_set_error("Unknown sequence_id " + std::to_string(sequence_id) + ".");
    return PKV_ERR_KEY;
  }
  *row_out = it->second.row;
  return PKV_OK;
}

int32_t pkv_allocator_decode_step(pkv_allocator* a, const int64_t* sequence_ids, int64_t n, int32_t* rows_out,
                                  int32_t* lens_out, int32_t* new_blocks_out, int32_t* token_blocks_out,
                                  int64_t* done) {
  pkv_clear_error();
  if (done) *done = 0;
  const bool cached = a->step_generation == a->generation && (int64_t)a->step_ids.size() == n &&
                      std::memcmp(a->step_ids.data(), sequence_ids, n * sizeof(int64_t)) == 0;
  if (!cached) {
    a->step_generation = ~0ull;
    a->step_ids.assign(sequence_ids, sequence_ids + n);
    a->step_seqs.assign(n, nullptr);
  }
  for (int64_t i = 0; i < n; ++i) {
    Sequence* sp = cached ? a->step_seqs[i] : nullptr;
    if (!sp) {
      auto it = a->seqs.find(sequence_ids[i]);
      if (it == a->seqs.end()) {
        pkv_set_error("Unknown sequence_id " + std::to_string(sequence_ids[i]) + ".");
        return PKV_ERR_KEY;
      }
      sp = &it->second;
      a->step_seqs[i] = sp;
    }
    Sequence& s = *sp;
    int32_t nb = -1;
    int32_t st = a->append(s, 1, /*track=*/false, &nb);
    if (st != PKV_OK) return st;
    rows_out[i] = s.row;
    lens_out[i] = (int32_t)s.tokens;
    new_blocks_out[i] = nb;
    if (token_blocks_out) token_blocks_out[i] = s.blocks.back();
    if (done) *done = i + 1;
  }
  a->step_generation = a->generation;
  return PKV_OK;
}

int32_t pkv_allocator_truncate(pkv_allocator* a, const int64_t* sequence_ids, const int64_t* token_counts,
                               int64_t n) {
  pkv_clear_error();
  for (int64_t i = 0; i < n; ++i) {
    if (token_counts[i] < 0) {
      pkv_set_error("token_count must be >= 0.");
      return PKV_ERR_VALUE;
    }
    auto it = a->seqs.find(sequence_ids[i]);
    if (it == a->seqs.end()) {
      pkv_set_error("Unknown sequence_id " + std::to_string(sequence_ids[i]) + ".");
      return PKV_ERR_KEY;
    }
    Sequence& s = it->second;
    if (token_counts[i] > s.tokens) {
      pkv_set_error("truncate cannot grow a sequence (" + std::to_string(token_counts[i]) + " > " +
                    std::to_string(s.tokens) + " tokens)");
      return PKV_ERR_VALUE;
    }
    const int64_t keep = a->required(token_counts[i]);
    while ((int64_t)s.blocks.size() > keep) {
      const int32_t b = s.blocks.back();
      s.blocks.pop_back();
      a->set_ref(b, a->refcount[b] - 1);
      if (a->refcount[b] == 0) a->set_free(b);
    }
    s.tokens = token_counts[i];
    a->mark_len(s.row);
  }
  return PKV_OK;
}

int32_t pkv_allocator_truncate_fill(pkv_allocator* a, const int64_t* sequence_ids, const int64_t* token_counts,
                                    int64_t n, int32_t* block_fill, int64_t fill_n) {
  pkv_clear_error();
  const int64_t bs = a->block_size;
  for (int64_t i = 0; i < n; ++i) {
    if (token_counts[i] < 0) {
      pkv_set_error("token_count must be >= 0.");
      return PKV_ERR_VALUE;
    }
    auto it = a->seqs.find(sequence_ids[i]);
    if (it == a->seqs.end()) {
      pkv_set_error("Unknown sequence_id " + std::to_string(sequence_ids[i]) + ".");
      return PKV_ERR_KEY;
    }
    Sequence& s = it->second;
    if (token_counts[i] > s.tokens) {
      pkv_set_error("truncate cannot grow a sequence (" + std::to_string(token_counts[i]) + " > " +
                    std::to_string(s.tokens) + " tokens)");
      return PKV_ERR_VALUE;
    }
    const int64_t keep = a->required(token_counts[i]);
    while ((int64_t)s.blocks.size() > keep) {
      const int32_t b = s.blocks.back();
      s.blocks.pop_back();
      a->set_ref(b, a->refcount[b] - 1);
      if (a->refcount[b] == 0) {
        a->set_free(b);
        if (block_fill && b >= 0 && b < fill_n) block_fill[b] = -1;
      }
    }
    s.tokens = token_counts[i];
    a->mark_len(s.row);
    const int32_t part = (int32_t)(token_counts[i] % bs);
    if (block_fill && keep > 0 && part) {
      const int32_t t = s.blocks.back();
      if (t >= 0 && t < fill_n && block_fill[t] > part) block_fill[t] = part;
    }
  }
  return PKV_OK;
}

int32_t pkv_allocator_token_counts(pkv_allocator* a, const int64_t* sequence_ids, int64_t n, int64_t* counts_out) {
  pkv_clear_error();
  for (int64_t i = 0; i < n; ++i) {
    auto it = a->seqs.find(sequence_ids[i]);
    if (it == a->seqs.end()) {
      pkv_set_error("Unknown sequence_id " + std::to_string(sequence_ids[i]) + ".");
      return PKV_ERR_KEY;
    }
    counts_out[i] = it->second.tokens;
  }
  return PKV_OK;
}

int32_t pkv_allocator_growth_blocks(pkv_allocator* a, const int64_t* sequence_ids, int64_t n, int32_t* need_out) {
  pkv_clear_error();
  const int64_t bs = a->block_size;
  for (int64_t i = 0; i < n; ++i) {
    auto it = a->seqs.find(sequence_ids[i]);
    if (it == a->seqs.end()) {
      pkv_set_error("Unknown sequence_id " + std::to_string(sequence_ids[i]) + ".");
      return PKV_ERR_KEY;
    }
    const Sequence& s = it->second;
    // One more token takes a fresh block at a block boundary, or a copy of a
    // partial tail block that forks still share; otherwise it fits in place.
    if ((int64_t)s.blocks.size() < a->required(s.tokens + 1)) {
      need_out[i] = 1;
    } else {
      need_out[i] = (s.tokens % bs != 0 && a->refcount[s.blocks.back()] > 1) ? 1 : 0;
    }
  }
  return PKV_OK;
}

int32_t pkv_allocator_chunk_slots(pkv_allocator* a, const int64_t* sequence_ids, const int64_t* q_lens, int64_t n,
                                  int32_t* rows_out, int32_t* past_out, int64_t* slots_out, int64_t slots_capacity,
                                  int32_t* block_fill, int64_t fill_n) {
  pkv_clear_error();
  const int64_t bs = a->block_size;
  int64_t k = 0;
  for (int64_t i = 0; i < n; ++i) {
    auto it = a->seqs.find(sequence_ids[i]);
    if (it == a->seqs.end()) {
      pkv_set_error("Unknown sequence_id " + std::to_string(sequence_ids[i]) + ".");
      return PKV_ERR_KEY;
    }
    const Sequence& s = it->second;
    if (q_lens[i] < 0 || q_lens[i] > s.tokens) {
      pkv_set_error("sequence " + std::to_string(sequence_ids[i]) + " holds " + std::to_string(s.tokens) +
                    " tokens, fewer than its chunk of " + std::to_string(q_lens[i]));
      return PKV_ERR_VALUE;
    }
    if (k + q_lens[i] > slots_capacity) {
      pkv_set_error("pkv_allocator_chunk_slots: slot buffer too small");
      return PKV_ERR_ARG;
    }
    rows_out[i] = s.row;
    const int64_t past = s.tokens - q_lens[i];
    past_out[i] = (int32_t)past;
    for (int64_t pos = past; pos < s.tokens; ++pos) {
      const int32_t blk = s.blocks[pos / bs];
      const int32_t in_blk = (int32_t)(pos % bs);
      slots_out[k++] = (int64_t)blk * bs + in_blk;
      if (block_fill && blk >= 0 && blk < fill_n && block_fill[blk] < in_blk + 1) block_fill[blk] = in_blk + 1;
    }
  }
  return PKV_OK;
}

int32_t pkv_allocator_touch_rows(pkv_allocator* a, const int32_t* rows, int64_t n) {
  pkv_clear_error();
  for (int64_t i = 0; i < n; ++i) {
    const int32_t r = rows[i];
    if (r < 0 || (size_t)r >= a->row_owner.size() || !a->row_owner[r]) continue;
    Sequence* s = a->row_owner[r];
    a->mark_len(r);
    if (!s->blocks.empty()) a->mark_entry(r, (int64_t)s->blocks.size() - 1);
  }
  return PKV_OK;
}

int32_t pkv_allocator_pending_updates(pkv_allocator* a, int64_t* n_table, int64_t* n_ref, int64_t* n_len,
                                      int64_t* n_copy) {
  *n_table = (int64_t)a->dirty_table.size();
  *n_ref = (int64_t)a->ref_dirty_list.size();
  *n_len = (int64_t)a->len_dirty_list.size();
  *n_copy = (int64_t)a->copies.size();
  return PKV_OK;
}

int32_t pkv_allocator_drain_updates(pkv_allocator* a, int32_t* out, int64_t capacity, int64_t* written) {
  pkv_clear_error();
  int64_t nt = 0;
  // Table entries: only live (row, col) pairs are emitted.
  std::vector<int32_t> table;
  table.reserve(a->dirty_table.size() * 3);
  for (uint64_t key : a->dirty_table) {
    int32_t row = (int32_t)(key >> 32);
    int32_t col = (int32_t)(key & 0xffffffffu);
    Sequence* s = (size_t)row < a->row_owner.size() ? a->row_owner[row] : nullptr;
    if (!s || col >= (int32_t)s->blocks.size()) continue;
    table.push_back(row);
    table.push_back(col);
    table.push_back(s->blocks[col]);
    ++nt;
  }
  int64_t nr = (int64_t)a->ref_dirty_list.size();
  int64_t nl = (int64_t)a->len_dirty_list.size();
  int64_t nc = (int64_t)a->copies.size();
  int64_t need = 4 + 3 * nt + 2 * nr + 2 * nl + 2 * nc;
  if (need > capacity) {
    pkv_set_error("update buffer too small: need " + std::to_string(need) + " int32");
    return PKV_ERR_ARG;
  }
  int32_t* p = out;
  *p++ = (int32_t)nt;
  *p++ = (int32_t)nr;
  *p++ = (int32_t)nl;
  *p++ = (int32_t)nc;
  std::memcpy(p, table.data(), sizeof(int32_t) * table.size());
  p += table.size();
  for (int32_t b : a->ref_dirty_list) {
    *p++ = b;
    *p++ = a->refcount[b];
    a->ref_dirty[b] = 0;
  }
  for (int32_t r : a->len_dirty_list) {
    Sequence* s = (size_t)r < a->row_owner.size() ? a->row_owner[r] : nullptr;
    *p++ = r;
    *p++ = s ? (int32_t)s->tokens : 0;
    a->len_dirty[r] = 0;
  }
  for (auto& c : a->copies) {
    *p++ = c.first;
    *p++ = c.second;
  }
  // clear() walks the whole bucket array, which keeps the size of the
  // largest batch of edits ever pending (tens of thousands after a bulk
  // placement): skip it when nothing is pending, and give the buckets back
  // after a large drain, so that a decode step's drain stays O(its updates).
  if (!a->dirty_table.empty()) {
    a->dirty_table.clear();
    if (a->dirty_table.bucket_count() > 4096) a->dirty_table.rehash(0);
  }
  a->ref_dirty_list.clear();
  a->len_dirty_list.clear();
  a->copies.clear();
  if (written) *written = need;
  return PKV_OK;
}

}  // extern "C"
