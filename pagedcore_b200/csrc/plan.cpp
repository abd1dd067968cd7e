// Piece tables of the split-K decode attention (host code, no device work).
//
// The batch's block tables form one flat list (row b owns blocks
// [prefix[b], prefix[b+1])).  The decode kernel runs one CTA per contiguous
// piece of it; a piece costs its blocks plus a row switch at every row that
// starts inside it (the kernel writes the finished row's output or partial
// and loads the next row's query before it streams on).  These tables cut
// the list so that every piece carries the same cost, optionally scaled by a
// per-piece speed weight, and tell the combine which pieces each row spans.

#include <cmath>
#include <cstdint>
#include <string>
#include <vector>

#include "pagedkv.h"
#include "status.h"

extern "C" int pkv_decode_tables(const int32_t *prefix, int32_t batch, int32_t grid, const float *weights,
                                 float row_cost, int32_t *pieces, int32_t *row_pieces) {
    pkv::clear_error();
    if (prefix == nullptr || pieces == nullptr || row_pieces == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "decode tables: null pointer argument");
    }
    if (batch < 1) return pkv::fail(PKV_VALUE_ERROR, "decode tables need a nonempty batch");
    if (prefix[0] != 0) return pkv::fail(PKV_VALUE_ERROR, "decode tables: prefix[0] must be 0");
    for (int32_t b = 0; b < batch; ++b) {
        if (prefix[b + 1] <= prefix[b]) {
            return pkv::fail(PKV_VALUE_ERROR, "decode tables: every row needs at least one block");
        }
    }
    const int32_t total = prefix[batch];
    if (grid < 1 || grid > total) {
        return pkv::fail(PKV_VALUE_ERROR, "decode tables: grid must lie in [1, " + std::to_string(total) + "]");
    }
    if (!(row_cost >= 0.0f) || !std::isfinite(row_cost)) {
        return pkv::fail(PKV_VALUE_ERROR, "decode tables: row_cost must be finite and non-negative");
    }
    double weight_sum = static_cast<double>(grid);
    if (weights != nullptr) {
        weight_sum = 0.0;
        for (int32_t g = 0; g < grid; ++g) {
            if (!(weights[g] > 0.0f) || !std::isfinite(weights[g])) {
                return pkv::fail(PKV_VALUE_ERROR, "decode tables: weights must be finite and positive");
            }
            weight_sum += weights[g];
        }
    }

    // Piece g begins at the first block where the cost of the blocks before
    // it reaches its share of the total cost.
    const double total_cost = static_cast<double>(total) + static_cast<double>(row_cost) * (batch - 1);
    std::vector<int32_t> begin(static_cast<size_t>(grid) + 1);
    begin[0] = 0;
    begin[grid] = total;
    double cost = 0.0, share = 0.0;
    int32_t x = 0, next_row = 1;  // prefix[next_row] is the next row start at or after x
    for (int32_t g = 1; g < grid; ++g) {
        share += weights != nullptr ? weights[g - 1] : 1.0;
        const double target = total_cost * share / weight_sum;
        while (x < total && cost < target) {
            while (next_row < batch && prefix[next_row] < x) ++next_row;
            cost += 1.0 + ((next_row < batch && prefix[next_row] == x) ? row_cost : 0.0);
            ++x;
        }
        begin[g] = x;
    }
    // Nonempty pieces: strictly increasing begins within [g, total - (grid - g)].
    for (int32_t g = 1; g < grid; ++g) {
        if (begin[g] <= begin[g - 1]) begin[g] = begin[g - 1] + 1;
    }
    for (int32_t g = grid - 1; g >= 1; --g) {
        if (begin[g] >= begin[g + 1]) begin[g] = begin[g + 1] - 1;
    }

    int32_t row = 0;
    for (int32_t g = 0; g < grid; ++g) {
        while (prefix[row + 1] <= begin[g]) ++row;
        pieces[4 * g + 0] = begin[g];
        pieces[4 * g + 1] = begin[g + 1];
        pieces[4 * g + 2] = row;
        pieces[4 * g + 3] = prefix[row];
    }
    int32_t piece = 0;
    for (int32_t b = 0; b < batch; ++b) {
        while (begin[piece + 1] <= prefix[b]) ++piece;
        int32_t last = piece;
        while (begin[last + 1] <= prefix[b + 1] - 1) ++last;
        row_pieces[2 * b + 0] = piece;
        row_pieces[2 * b + 1] = last;
    }
    return PKV_OK;
}
