// Block ledger of the paged KV cache: the host-side bookkeeping of
// PagedCore's KVAllocator (src/pagedcore/kv_cache.py:63-357), as an O(1)
// C++ structure behind the C ABI of include/pagedkv.h.
//
// The block-assignment order is part of the contract (tests pin tables such
// as (0, 2, 3) and (2, 0, 3, 4)), so the free list is the same LIFO stack as
// the reference's `_free_blocks` list: back() is the top, new blocks are
// taken from the top, and release pushes a table in reverse so that its first
// block ends on top.  Credits, staged decode and all error classes/messages
// follow the reference; the only structural change is that the reference's
// O(pool) re-validation on every call is optional (PKV_VALIDATE_FULL) and an
// incremental check of the touched requests is the fast mode.

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "pagedkv.h"
#include "status.h"

namespace {

constexpr int32_t kBlockTokens = PKV_BLOCK_TOKENS;
constexpr int32_t kContextLimit = PKV_CONTEXT_LIMIT;
constexpr int64_t kMaxCredits = PKV_MAX_CREDITS;
constexpr int32_t kLayers = PKV_LAYERS;

inline int32_t blocks_for(int64_t length) {
    return static_cast<int32_t>((length + kBlockTokens - 1) / kBlockTokens);
}

struct Sequence {
    int64_t credits = 0;
    std::vector<int32_t> blocks;
    int32_t length = 0;
};

}  // namespace

struct pkv_ledger {
    int32_t num_blocks = 0;
    int32_t validation = PKV_VALIDATE_FULL;
    std::vector<int32_t> free_stack;    // bottom .. top (back)
    std::vector<int64_t> owner;         // per block: owning request, or kNoOwner
    std::unordered_map<int64_t, Sequence> sequences;
    // Counters kept in O(1); FULL validation recomputes and compares them.
    int64_t reserved = 0;
    int64_t owned = 0;
    int64_t live = 0;

    // Staged decode (kv_cache.py:181-219).
    bool staging = false;
    std::vector<int64_t> staged_requests;
    std::vector<int32_t> staged_new_block;  // -1 when the row reuses its last block
    std::vector<int32_t> staged_written;
    std::unordered_map<int64_t, int32_t> staged_row;
    int32_t staged_additional = 0;

    static constexpr int64_t kNoOwner = INT64_MIN;
};

namespace {

using pkv::fail;

// kv_cache.py:314-357, in the reference's order of checks.
int audit_full(pkv_ledger *L) {
    const int32_t n = L->num_blocks;
    for (const auto &entry : L->sequences) {
        const Sequence &s = entry.second;
        if (s.length < 0 || s.length > kContextLimit ||
            static_cast<int64_t>(s.blocks.size()) != blocks_for(s.length) ||
            !(static_cast<int64_t>(s.blocks.size()) <= s.credits && s.credits <= kMaxCredits)) {
            return fail(PKV_RUNTIME_ERROR, "corrupt KV block table or reservation");
        }
    }
    for (int32_t b : L->free_stack) {
        if (b < 0 || b >= n) return fail(PKV_RUNTIME_ERROR, "invalid physical KV block");
    }
    for (const auto &entry : L->sequences) {
        for (int32_t b : entry.second.blocks) {
            if (b < 0 || b >= n) return fail(PKV_RUNTIME_ERROR, "invalid physical KV block");
        }
    }
    // Ownership derived from the tables, compared with the recorded owners.
    std::vector<int64_t> derived(static_cast<size_t>(n), pkv_ledger::kNoOwner);
    int64_t assigned = 0;
    bool duplicate = false;
    for (const auto &entry : L->sequences) {
        for (int32_t b : entry.second.blocks) {
            ++assigned;
            if (derived[b] != pkv_ledger::kNoOwner) duplicate = true;
            derived[b] = entry.first;
        }
    }
    if (duplicate) return fail(PKV_RUNTIME_ERROR, "physical KV blocks must have unique owners");
    std::vector<uint8_t> in_free(static_cast<size_t>(n), 0);
    for (int32_t b : L->free_stack) {
        if (in_free[b]) return fail(PKV_RUNTIME_ERROR, "free KV blocks must be unique");
        in_free[b] = 1;
    }
    for (int32_t b = 0; b < n; ++b) {
        if (in_free[b] && derived[b] != pkv_ledger::kNoOwner) {
            return fail(PKV_RUNTIME_ERROR, "owned KV blocks must not be free");
        }
    }
    if (static_cast<int64_t>(L->free_stack.size()) + assigned != n) {
        return fail(PKV_RUNTIME_ERROR, "KV blocks must cover the pool");
    }
    for (int32_t b = 0; b < n; ++b) {
        if (derived[b] != L->owner[b]) {
            return fail(PKV_RUNTIME_ERROR, "KV blocks are not owned by the recorded requests");
        }
    }
    int64_t reserved = 0, live = 0;
    for (const auto &entry : L->sequences) {
        reserved += entry.second.credits;
        live += entry.second.length;
    }
    if (reserved != L->reserved || live != L->live || assigned != L->owned) {
        return fail(PKV_RUNTIME_ERROR, "corrupt KV block table or reservation");
    }
    return PKV_OK;
}

// The part of the audit that concerns one request: its own table shape and
// the ownership of its blocks.  Used by the INCREMENTAL mode.
int audit_request(pkv_ledger *L, int64_t request, const Sequence &s) {
    if (s.length < 0 || s.length > kContextLimit ||
        static_cast<int64_t>(s.blocks.size()) != blocks_for(s.length) ||
        !(static_cast<int64_t>(s.blocks.size()) <= s.credits && s.credits <= kMaxCredits)) {
        return fail(PKV_RUNTIME_ERROR, "corrupt KV block table or reservation");
    }
    for (int32_t b : s.blocks) {
        if (b < 0 || b >= L->num_blocks) return fail(PKV_RUNTIME_ERROR, "invalid physical KV block");
        if (L->owner[b] != request) {
            return fail(PKV_RUNTIME_ERROR, "KV blocks are not owned by the recorded requests");
        }
    }
    return PKV_OK;
}

// Audit before/after a call: the whole ledger in FULL mode, else the
// requests the call touches (`request` may be absent from the map).
int audit(pkv_ledger *L, const int64_t *requests = nullptr, int32_t count = 0) {
    if (L->validation == PKV_VALIDATE_FULL) return audit_full(L);
    for (int32_t i = 0; i < count; ++i) {
        auto it = L->sequences.find(requests[i]);
        if (it == L->sequences.end()) continue;
        int rc = audit_request(L, it->first, it->second);
        if (rc) return rc;
    }
    return PKV_OK;
}

int check_mutation(pkv_ledger *L) {
    if (L->staging) {
        return fail(PKV_RUNTIME_ERROR, "KV mutation is not allowed during a staged decode append");
    }
    return PKV_OK;
}

int key_error(int64_t request) {
    return fail(PKV_KEY_ERROR, "unknown KV request " + std::to_string(request));
}

// The (blocks, length) a request exposes to readers at `layer`
// (kv_cache.py:256-263); layer -1 means the committed view and
// PKV_VIEW_STAGED the staged view whatever layers were written.
int resolve_view(pkv_ledger *L, int64_t request, int32_t layer, const Sequence **seq,
                 int32_t *new_block, int32_t *length) {
    auto it = L->sequences.find(request);
    if (it == L->sequences.end()) return key_error(request);
    *seq = &it->second;
    *new_block = -1;
    *length = it->second.length;
    if ((layer >= 0 || layer == PKV_VIEW_STAGED) && L->staging) {
        auto row = L->staged_row.find(request);
        if (row != L->staged_row.end()) {
            if (layer != PKV_VIEW_STAGED && layer >= L->staged_written[row->second]) {
                return fail(PKV_RUNTIME_ERROR, "cannot read an unwritten decode layer");
            }
            *new_block = L->staged_new_block[row->second];
            *length = it->second.length + 1;
        }
    }
    return PKV_OK;
}

}  // namespace

extern "C" {

int pkv_abi_version(void) { return PKV_ABI_VERSION; }

int pkv_ledger_new(int32_t num_blocks, int32_t validation, pkv_ledger **out) {
    pkv::clear_error();
    if (out == nullptr) return fail(PKV_VALUE_ERROR, "output pointer must not be NULL");
    *out = nullptr;
    if (num_blocks < 1) {
        return fail(PKV_VALUE_ERROR,
                    "KV pool must be contiguous FP16 [22, 2, blocks, 16, 4, 64] storage");
    }
    if (validation != PKV_VALIDATE_FULL && validation != PKV_VALIDATE_INCREMENTAL) {
        return fail(PKV_VALUE_ERROR, "unknown validation level");
    }
    auto *L = new pkv_ledger();
    L->num_blocks = num_blocks;
    L->validation = validation;
    L->free_stack.resize(static_cast<size_t>(num_blocks));
    // kv_cache.py:86: [N-1, ..., 1, 0] with 0 on top.
    for (int32_t i = 0; i < num_blocks; ++i) L->free_stack[i] = num_blocks - 1 - i;
    L->owner.assign(static_cast<size_t>(num_blocks), pkv_ledger::kNoOwner);
    *out = L;
    return PKV_OK;
}

void pkv_ledger_free(pkv_ledger *ledger) { delete ledger; }

int pkv_ledger_set_validation(pkv_ledger *L, int32_t validation) {
    pkv::clear_error();
    if (validation != PKV_VALIDATE_FULL && validation != PKV_VALIDATE_INCREMENTAL) {
        return fail(PKV_VALUE_ERROR, "unknown validation level");
    }
    L->validation = validation;
    return PKV_OK;
}

int pkv_ledger_reserve(pkv_ledger *L, int64_t request, int64_t credits) {
    pkv::clear_error();
    int rc = check_mutation(L);
    if (rc) return rc;
    if (credits <= 0) return fail(PKV_VALUE_ERROR, "maximum_block_credits must be a positive integer");
    if (L->sequences.count(request)) return fail(PKV_VALUE_ERROR, "request already has a KV cache");
    if ((rc = audit(L))) return rc;  // the reference's capacity() call
    if (credits > L->num_blocks) return fail(PKV_VALUE_ERROR, "reservation exceeds total KV pool capacity");
    if (credits > kMaxCredits) return fail(PKV_VALUE_ERROR, "reservation exceeds KV context capacity");
    if (credits > L->num_blocks - L->reserved) {
        return fail(PKV_RUNTIME_ERROR, "KV pool has insufficient unreserved blocks");
    }
    Sequence s;
    s.credits = credits;
    L->sequences.emplace(request, std::move(s));
    L->reserved += credits;
    return audit(L, &request, 1);
}

int pkv_ledger_release(pkv_ledger *L, int64_t request) {
    pkv::clear_error();
    int rc = check_mutation(L);
    if (rc) return rc;
    if ((rc = audit(L, &request, 1))) return rc;
    auto it = L->sequences.find(request);
    if (it == L->sequences.end()) return key_error(request);
    Sequence &s = it->second;
    for (int32_t b : s.blocks) L->owner[b] = pkv_ledger::kNoOwner;
    // kv_cache.py:297: extend(reversed(blocks)) puts blocks[0] on top.
    for (auto b = s.blocks.rbegin(); b != s.blocks.rend(); ++b) L->free_stack.push_back(*b);
    L->owned -= static_cast<int64_t>(s.blocks.size());
    L->reserved -= s.credits;
    L->live -= s.length;
    L->sequences.erase(it);
    return audit(L);
}

int pkv_ledger_capacity(pkv_ledger *L, int64_t out[6]) {
    pkv::clear_error();
    int rc = audit(L);
    if (rc) return rc;
    out[0] = L->num_blocks;
    out[1] = static_cast<int64_t>(L->free_stack.size());
    out[2] = L->owned;
    out[3] = L->reserved;
    out[4] = static_cast<int64_t>(L->sequences.size());
    out[5] = L->live;
    return PKV_OK;
}

int pkv_ledger_length(pkv_ledger *L, int64_t request, int32_t *out_length) {
    pkv::clear_error();
    int rc = audit(L, &request, 1);
    if (rc) return rc;
    auto it = L->sequences.find(request);
    if (it == L->sequences.end()) return key_error(request);
    *out_length = it->second.length;
    return PKV_OK;
}

int pkv_ledger_table(pkv_ledger *L, int64_t request, int32_t *out_blocks, int32_t capacity,
                     int32_t *out_count) {
    pkv::clear_error();
    int rc = audit(L, &request, 1);
    if (rc) return rc;
    auto it = L->sequences.find(request);
    if (it == L->sequences.end()) return key_error(request);
    const auto &blocks = it->second.blocks;
    *out_count = static_cast<int32_t>(blocks.size());
    if (static_cast<int32_t>(blocks.size()) > capacity) {
        return fail(PKV_VALUE_ERROR, "block table buffer is too small");
    }
    std::copy(blocks.begin(), blocks.end(), out_blocks);
    return PKV_OK;
}

int pkv_ledger_append_plan(pkv_ledger *L, int64_t request, int32_t tokens, int32_t *out_slots,
                           int32_t *out_start_position) {
    pkv::clear_error();
    int rc = check_mutation(L);
    if (rc) return rc;
    if ((rc = audit(L, &request, 1))) return rc;
    auto it = L->sequences.find(request);
    if (it == L->sequences.end()) return key_error(request);
    const Sequence &s = it->second;
    if (tokens < 1) {
        return fail(PKV_VALUE_ERROR, "K and V must share FP16 [22, tokens, 4, 64] on the pool device");
    }
    const int64_t length = static_cast<int64_t>(s.length) + tokens;
    if (length > kContextLimit) return fail(PKV_VALUE_ERROR, "KV cache must not exceed 2048 token positions");
    const int32_t required = blocks_for(length);
    if (required > s.credits) return fail(PKV_RUNTIME_ERROR, "KV append exceeds request reservation");
    const int32_t additional = required - static_cast<int32_t>(s.blocks.size());
    if (additional > static_cast<int32_t>(L->free_stack.size())) {
        return fail(PKV_RUNTIME_ERROR, "KV pool has insufficient free blocks");
    }
    // kv_cache.py:158: new blocks are reversed(free[-additional:]).
    const size_t top = L->free_stack.size();
    for (int32_t t = 0; t < tokens; ++t) {
        const int32_t position = s.length + t;
        const int32_t logical = position / kBlockTokens;
        const int32_t physical =
            logical < static_cast<int32_t>(s.blocks.size())
                ? s.blocks[logical]
                : L->free_stack[top - 1 - (logical - s.blocks.size())];
        out_slots[t] = physical * kBlockTokens + position % kBlockTokens;
    }
    if (out_start_position) *out_start_position = s.length;
    return PKV_OK;
}

int pkv_ledger_append_commit(pkv_ledger *L, int64_t request, int32_t tokens) {
    pkv::clear_error();
    int rc = check_mutation(L);
    if (rc) return rc;
    auto it = L->sequences.find(request);
    if (it == L->sequences.end()) return key_error(request);
    Sequence &s = it->second;
    const int64_t length = static_cast<int64_t>(s.length) + tokens;
    if (tokens < 1 || length > kContextLimit) return fail(PKV_VALUE_ERROR, "invalid KV append commit");
    const int32_t required = blocks_for(length);
    const int32_t additional = required - static_cast<int32_t>(s.blocks.size());
    if (required > s.credits || additional > static_cast<int32_t>(L->free_stack.size())) {
        return fail(PKV_RUNTIME_ERROR, "KV append exceeds request reservation");
    }
    // kv_cache.py:175-178: pop the new blocks (top first) and publish.
    for (int32_t i = 0; i < additional; ++i) {
        const int32_t b = L->free_stack.back();
        L->free_stack.pop_back();
        s.blocks.push_back(b);
        L->owner[b] = request;
    }
    L->owned += additional;
    L->live += tokens;
    s.length = static_cast<int32_t>(length);
    return audit(L, &request, 1);
}

// Several appends in one call: request i is planned as if requests 0..i-1 of
// the call had been committed before it, so its new blocks continue down the
// free stack below theirs (the order in which sequential appends would take
// them).  Nothing changes until commit_many, which checks every request
// before it changes any.
namespace {

int check_distinct(const int64_t *requests, int32_t count) {
    std::unordered_set<int64_t> seen;
    for (int32_t i = 0; i < count; ++i) {
        if (!seen.insert(requests[i]).second) {
            return fail(PKV_VALUE_ERROR, "a request may appear only once in a batched append");
        }
    }
    return PKV_OK;
}

}  // namespace

int pkv_ledger_append_plan_many(pkv_ledger *L, const int64_t *requests, const int32_t *tokens, int32_t count,
                                int32_t *out_slots, int32_t *out_start_positions) {
    pkv::clear_error();
    int rc = check_mutation(L);
    if (rc) return rc;
    if (count < 1) return fail(PKV_VALUE_ERROR, "a batched append needs at least one request");
    if ((rc = check_distinct(requests, count))) return rc;
    if ((rc = audit(L, requests, count))) return rc;
    const size_t top = L->free_stack.size();
    size_t taken = 0;  // blocks the earlier requests of this call take from the top
    int64_t at = 0;
    for (int32_t i = 0; i < count; ++i) {
        auto it = L->sequences.find(requests[i]);
        if (it == L->sequences.end()) return key_error(requests[i]);
        const Sequence &s = it->second;
        if (tokens[i] < 1) {
            return fail(PKV_VALUE_ERROR, "K and V must share FP16 [22, tokens, 4, 64] on the pool device");
        }
        const int64_t length = static_cast<int64_t>(s.length) + tokens[i];
        if (length > kContextLimit) return fail(PKV_VALUE_ERROR, "KV cache must not exceed 2048 token positions");
        const int32_t required = blocks_for(length);
        if (required > s.credits) return fail(PKV_RUNTIME_ERROR, "KV append exceeds request reservation");
        const int32_t additional = required - static_cast<int32_t>(s.blocks.size());
        if (static_cast<size_t>(additional) > top - taken) {
            return fail(PKV_RUNTIME_ERROR, "KV pool has insufficient free blocks");
        }
        for (int32_t t = 0; t < tokens[i]; ++t) {
            const int32_t position = s.length + t;
            const int32_t logical = position / kBlockTokens;
            const int32_t physical =
                logical < static_cast<int32_t>(s.blocks.size())
                    ? s.blocks[logical]
                    : L->free_stack[top - 1 - taken - (logical - s.blocks.size())];
            out_slots[at + t] = physical * kBlockTokens + position % kBlockTokens;
        }
        if (out_start_positions) out_start_positions[i] = s.length;
        taken += additional;
        at += tokens[i];
    }
    return PKV_OK;
}

int pkv_ledger_append_commit_many(pkv_ledger *L, const int64_t *requests, const int32_t *tokens, int32_t count) {
    pkv::clear_error();
    int rc = check_mutation(L);
    if (rc) return rc;
    if (count < 1) return fail(PKV_VALUE_ERROR, "a batched append needs at least one request");
    if ((rc = check_distinct(requests, count))) return rc;
    size_t taken = 0;
    for (int32_t i = 0; i < count; ++i) {
        auto it = L->sequences.find(requests[i]);
        if (it == L->sequences.end()) return key_error(requests[i]);
        const Sequence &s = it->second;
        const int64_t length = static_cast<int64_t>(s.length) + tokens[i];
        if (tokens[i] < 1 || length > kContextLimit) return fail(PKV_VALUE_ERROR, "invalid KV append commit");
        const int32_t required = blocks_for(length);
        const int32_t additional = required - static_cast<int32_t>(s.blocks.size());
        if (required > s.credits || static_cast<size_t>(additional) > L->free_stack.size() - taken) {
            return fail(PKV_RUNTIME_ERROR, "KV append exceeds request reservation");
        }
        taken += additional;
    }
    for (int32_t i = 0; i < count; ++i) {
        Sequence &s = L->sequences.find(requests[i])->second;
        const int64_t length = static_cast<int64_t>(s.length) + tokens[i];
        const int32_t additional = blocks_for(length) - static_cast<int32_t>(s.blocks.size());
        // kv_cache.py:175-178 for each request in order: pop its new blocks (top first).
        for (int32_t b = 0; b < additional; ++b) {
            const int32_t block = L->free_stack.back();
            L->free_stack.pop_back();
            s.blocks.push_back(block);
            L->owner[block] = requests[i];
        }
        L->owned += additional;
        L->live += tokens[i];
        s.length = static_cast<int32_t>(length);
    }
    return audit(L, requests, count);
}

int pkv_ledger_decode_begin(pkv_ledger *L, const int64_t *requests, int32_t count,
                            int32_t *out_slots, int32_t *out_positions) {
    pkv::clear_error();
    int rc = check_mutation(L);
    if (rc) return rc;
    if ((rc = audit(L, requests, count))) return rc;
    if (count < 1) return fail(PKV_VALUE_ERROR, "decode requires nonempty, distinct request IDs");
    std::unordered_map<int64_t, int32_t> rows;
    rows.reserve(static_cast<size_t>(count) * 2);
    for (int32_t i = 0; i < count; ++i) {
        if (!rows.emplace(requests[i], i).second) {
            return fail(PKV_VALUE_ERROR, "decode requires nonempty, distinct request IDs");
        }
    }
    std::vector<int32_t> new_block(static_cast<size_t>(count), -1);
    int32_t additional = 0;
    const size_t top = L->free_stack.size();
    for (int32_t i = 0; i < count; ++i) {
        auto it = L->sequences.find(requests[i]);
        if (it == L->sequences.end()) return key_error(requests[i]);
        const Sequence &s = it->second;
        if (!(1 <= s.length && s.length < kContextLimit)) {
            return fail(PKV_VALUE_ERROR, "decode requires 1 to 2047 cached token positions");
        }
        if (blocks_for(static_cast<int64_t>(s.length) + 1) > s.credits) {
            return fail(PKV_RUNTIME_ERROR, "KV append exceeds request reservation");
        }
        if (s.length % kBlockTokens == 0) {
            ++additional;
            if (additional > static_cast<int32_t>(top)) {
                return fail(PKV_RUNTIME_ERROR, "KV pool has insufficient free blocks");
            }
            new_block[i] = L->free_stack[top - additional];  // free[-additional]
        }
    }
    for (int32_t i = 0; i < count; ++i) {
        const Sequence &s = L->sequences.find(requests[i])->second;
        const int32_t physical = new_block[i] >= 0 ? new_block[i] : s.blocks[s.length / kBlockTokens];
        if (out_slots) out_slots[i] = physical * kBlockTokens + s.length % kBlockTokens;
        if (out_positions) out_positions[i] = s.length;
    }
    L->staging = true;
    L->staged_requests.assign(requests, requests + count);
    L->staged_new_block = std::move(new_block);
    L->staged_written.assign(static_cast<size_t>(count), 0);
    L->staged_row = std::move(rows);
    L->staged_additional = additional;
    return PKV_OK;
}

namespace {
int decode_row_check(pkv_ledger *L, int32_t row, int32_t layer) {
    if (layer < 0 || layer >= kLayers) {
        return fail(PKV_VALUE_ERROR, "layer_index must identify one of the 22 decoder layers");
    }
    if (layer != L->staged_written[row]) {
        return fail(PKV_VALUE_ERROR, "decode cache layers must be written once in order");
    }
    return PKV_OK;
}

void decode_row_slot(pkv_ledger *L, int32_t row, int32_t *slot, int32_t *position) {
    const Sequence &s = L->sequences.find(L->staged_requests[row])->second;
    const int32_t nb = L->staged_new_block[row];
    const int32_t physical = nb >= 0 ? nb : s.blocks[s.length / kBlockTokens];
    if (slot) *slot = physical * kBlockTokens + s.length % kBlockTokens;
    if (position) *position = s.length;
}
}  // namespace

int pkv_ledger_decode_check(pkv_ledger *L, int64_t request, int32_t layer, int32_t *out_slot,
                            int32_t *out_position) {
    pkv::clear_error();
    int rc = audit(L);
    if (rc) return rc;
    if (!L->staging) return fail(PKV_RUNTIME_ERROR, "decode writes require a staged append");
    if (request == -1) {
        for (int32_t row = 0; row < static_cast<int32_t>(L->staged_requests.size()); ++row) {
            if ((rc = decode_row_check(L, row, layer))) return rc;
        }
        return PKV_OK;
    }
    auto row = L->staged_row.find(request);
    if (row == L->staged_row.end()) return key_error(request);
    if ((rc = decode_row_check(L, row->second, layer))) return rc;
    decode_row_slot(L, row->second, out_slot, out_position);
    return PKV_OK;
}

int pkv_ledger_decode_mark(pkv_ledger *L, int64_t request, int32_t layer) {
    pkv::clear_error();
    if (!L->staging) return fail(PKV_RUNTIME_ERROR, "decode writes require a staged append");
    if (request == -1) {
        for (int32_t row = 0; row < static_cast<int32_t>(L->staged_requests.size()); ++row) {
            int rc = decode_row_check(L, row, layer);
            if (rc) return rc;
        }
        for (auto &w : L->staged_written) w = layer + 1;
        return PKV_OK;
    }
    auto row = L->staged_row.find(request);
    if (row == L->staged_row.end()) return key_error(request);
    int rc = decode_row_check(L, row->second, layer);
    if (rc) return rc;
    L->staged_written[row->second] = layer + 1;
    return PKV_OK;
}

int pkv_ledger_decode_mark_layers(pkv_ledger *L, int32_t first, int32_t count) {
    pkv::clear_error();
    int rc = audit(L);
    if (rc) return rc;
    if (!L->staging) return fail(PKV_RUNTIME_ERROR, "decode writes require a staged append");
    if (count < 1 || first < 0 || first + count > kLayers) {
        return fail(PKV_VALUE_ERROR, "layer_index must identify one of the 22 decoder layers");
    }
    for (int32_t row = 0; row < static_cast<int32_t>(L->staged_requests.size()); ++row) {
        if ((rc = decode_row_check(L, row, first))) return rc;
    }
    for (auto &w : L->staged_written) w = first + count;
    return PKV_OK;
}

void pkv_ledger_decode_abort(pkv_ledger *L) {
    L->staging = false;
    L->staged_requests.clear();
    L->staged_new_block.clear();
    L->staged_written.clear();
    L->staged_row.clear();
    L->staged_additional = 0;
}

int pkv_ledger_decode_commit(pkv_ledger *L) {
    pkv::clear_error();
    if (!L->staging) return fail(PKV_RUNTIME_ERROR, "decode writes require a staged append");
    for (int32_t w : L->staged_written) {
        if (w != kLayers) {
            pkv_ledger_decode_abort(L);
            return fail(PKV_RUNTIME_ERROR, "decode must write every cache layer before committing");
        }
    }
    // kv_cache.py:210-216: delete free[-additional:], then publish each row.
    L->free_stack.resize(L->free_stack.size() - L->staged_additional);
    const int32_t count = static_cast<int32_t>(L->staged_requests.size());
    for (int32_t i = 0; i < count; ++i) {
        const int64_t request = L->staged_requests[i];
        Sequence &s = L->sequences.find(request)->second;
        if (L->staged_new_block[i] >= 0) {
            s.blocks.push_back(L->staged_new_block[i]);
            L->owner[L->staged_new_block[i]] = request;
            ++L->owned;
        }
        s.length += 1;
        ++L->live;
    }
    std::vector<int64_t> touched = L->staged_requests;
    pkv_ledger_decode_abort(L);
    return audit(L, touched.data(), static_cast<int32_t>(touched.size()));
}

int pkv_ledger_decode_active(pkv_ledger *L) { return L->staging ? 1 : 0; }

int pkv_ledger_view(pkv_ledger *L, int64_t request, int32_t layer, int32_t *out_blocks,
                    int32_t capacity, int32_t *out_count, int32_t *out_length) {
    pkv::clear_error();
    int rc = audit(L, &request, 1);
    if (rc) return rc;
    const Sequence *s = nullptr;
    int32_t new_block = -1, length = 0;
    if ((rc = resolve_view(L, request, layer, &s, &new_block, &length))) return rc;
    const int32_t count = static_cast<int32_t>(s->blocks.size()) + (new_block >= 0 ? 1 : 0);
    *out_count = count;
    *out_length = length;
    if (count > capacity) return fail(PKV_VALUE_ERROR, "block table buffer is too small");
    std::copy(s->blocks.begin(), s->blocks.end(), out_blocks);
    if (new_block >= 0) out_blocks[count - 1] = new_block;
    return PKV_OK;
}

int pkv_ledger_batch(pkv_ledger *L, const int64_t *requests, int32_t count, int32_t layer,
                     int32_t *out_lengths, int32_t *out_prefix, int32_t *out_flat,
                     int32_t flat_capacity, int32_t *out_total_blocks) {
    pkv::clear_error();
    int rc = audit(L, requests, count);
    if (rc) return rc;
    if ((layer < 0 || layer >= kLayers) && layer != PKV_VIEW_STAGED) {
        return fail(PKV_VALUE_ERROR, "layer_index must identify one of the 22 decoder layers");
    }
    int32_t total = 0;
    out_prefix[0] = 0;
    for (int32_t i = 0; i < count; ++i) {
        const Sequence *s = nullptr;
        int32_t new_block = -1, length = 0;
        if ((rc = resolve_view(L, requests[i], layer, &s, &new_block, &length))) return rc;
        if (length == 0) return fail(PKV_VALUE_ERROR, "attention requires a nonempty cache");
        const int32_t nb = static_cast<int32_t>(s->blocks.size()) + (new_block >= 0 ? 1 : 0);
        if (total + nb > flat_capacity) return fail(PKV_VALUE_ERROR, "block table buffer is too small");
        std::copy(s->blocks.begin(), s->blocks.end(), out_flat + total);
        if (new_block >= 0) out_flat[total + nb - 1] = new_block;
        total += nb;
        out_lengths[i] = length;
        out_prefix[i + 1] = total;
    }
    *out_total_blocks = total;
    return PKV_OK;
}

int pkv_ledger_audit(pkv_ledger *L) {
    pkv::clear_error();
    return audit_full(L);
}

int pkv_ledger_free_list(pkv_ledger *L, int32_t *out, int32_t capacity, int32_t *out_count) {
    pkv::clear_error();
    *out_count = static_cast<int32_t>(L->free_stack.size());
    if (*out_count > capacity) return fail(PKV_VALUE_ERROR, "free list buffer is too small");
    std::copy(L->free_stack.begin(), L->free_stack.end(), out);
    return PKV_OK;
}

int pkv_ledger_reorder_free(pkv_ledger *L, const int32_t *blocks, int32_t count) {
    pkv::clear_error();
    int rc = check_mutation(L);
    if (rc) return rc;
    if (count != static_cast<int32_t>(L->free_stack.size())) {
        return fail(PKV_VALUE_ERROR, "free-list order must be a permutation of the free blocks");
    }
    std::vector<uint8_t> seen(static_cast<size_t>(L->num_blocks), 0);
    for (int32_t b : L->free_stack) seen[b] = 1;
    for (int32_t i = 0; i < count; ++i) {
        const int32_t b = blocks[i];
        if (b < 0 || b >= L->num_blocks || seen[b] != 1) {
            return fail(PKV_VALUE_ERROR, "free-list order must be a permutation of the free blocks");
        }
        seen[b] = 2;
    }
    L->free_stack.assign(blocks, blocks + count);
    return audit(L);
}

int pkv_ledger_debug_set_table(pkv_ledger *L, int64_t request, const int32_t *blocks,
                               int32_t count, int32_t length) {
    pkv::clear_error();
    auto it = L->sequences.find(request);
    if (it == L->sequences.end()) return key_error(request);
    Sequence &s = it->second;
    L->owned += count - static_cast<int64_t>(s.blocks.size());
    L->live += static_cast<int64_t>(length) - s.length;
    s.blocks.assign(blocks, blocks + count);
    s.length = length;
    return PKV_OK;
}

int pkv_ledger_debug_set_free(pkv_ledger *L, const int32_t *blocks, int32_t count) {
    pkv::clear_error();
    L->free_stack.assign(blocks, blocks + count);
    return PKV_OK;
}

}  // extern "C"
