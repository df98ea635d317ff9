// Host-side planning of a paged-attention launch: chunks of consecutive rows
// of one sequence for the chunk kernel where it applies, and for every other
// row one work item, or several (split-KV) for rows whose visible range is
// long relative to the batch, so that the grid covers every SM; split rows
// get a combine entry.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <utility>
#include <vector>

namespace tvara {

struct AttnPlan {
    std::vector<int4> work;   // {row, table offset, pos begin, pos end}
    std::vector<int> part;    // partial slot or -1
    std::vector<int4> comb;   // {row, first part, parts, 0}
    std::vector<int4> chunk;  // {first row, table offset, visible of the first row, rows}
    int parts = 0;
};

// Runs of consecutive rows that belong to one sequence (same table offset)
// and see one more position each: the rows of a prefill chunk or of a
// speculative verify.  Returns {first row, length} pairs.
inline std::vector<std::pair<int, int>> row_runs(const std::vector<int>& visible, const std::vector<int>& table_off) {
    std::vector<std::pair<int, int>> runs;
    for (int t = 0; t < int(visible.size());) {
        int n = 1;
        while (t + n < int(visible.size()) && table_off[t + n] == table_off[t] && visible[t + n] == visible[t] + n) ++n;
        runs.emplace_back(t, n);
        t += n;
    }
    return runs;
}

// chunk_rows > 0: runs of at least two rows go to the chunk kernel in pieces
// of up to chunk_rows rows (each reads its sequence's K/V once for all its
// rows) when that gives a grid of at least one CTA per SM or the run is a
// prefill-sized one (>= chunk_rows rows); every other row is planned for the
// per-row kernels below.
inline AttnPlan plan_attention(const std::vector<int>& visible, const std::vector<int>& table_off, int tpb, int kv_heads,
                               std::size_t parts_cap, int sms = 148, int chunk_rows = 0) {
    AttnPlan plan;
    std::vector<char> chunked(visible.size(), 0);
    if (chunk_rows > 1) {
        const auto runs = row_runs(visible, table_off);
        long long pieces = 0;
        for (const auto& r : runs)
            if (r.second > 1) pieces += (r.second + chunk_rows - 1) / chunk_rows;
        for (const auto& [first, n] : runs) {
            if (n < 2 || (pieces * kv_heads < sms && n < chunk_rows)) continue;
            for (int k = 0; k < n; k += chunk_rows) {
                const int rows = std::min(chunk_rows, n - k);
                plan.chunk.push_back(make_int4(first + k, table_off[first], visible[first + k], rows));
            }
            for (int k = 0; k < n; ++k) chunked[first + k] = 1;
        }
    }
    long long total = 0;
    for (std::size_t t = 0; t < visible.size(); ++t)
        if (!chunked[t]) total += visible[t];
    const long long target = std::max<long long>(1, (long long)sms * 8 / std::max(1, kv_heads));
    long long P = std::max<long long>((long long)tpb * 8, (total + target - 1) / target);
    P = (P + tpb - 1) / tpb * tpb;
    auto count = [&](long long p) {
        long long n = 0;
        for (std::size_t t = 0; t < visible.size(); ++t)
            if (!chunked[t] && visible[t] > p) n += (visible[t] + p - 1) / p;
        return n;
    };
    while (count(P) > (long long)parts_cap) P *= 2;
    for (std::size_t t = 0; t < visible.size(); ++t) {
        if (chunked[t]) continue;
        const int vis = visible[t];
        if (vis <= P) {
            plan.work.push_back(make_int4(int(t), table_off[t], 0, vis));
            plan.part.push_back(-1);
        } else {
            const int np = int((vis + P - 1) / P);
            plan.comb.push_back(make_int4(int(t), plan.parts, np, 0));
            for (int k = 0; k < np; ++k) {
                plan.work.push_back(make_int4(int(t), table_off[t], int(k * P), int(std::min<long long>((k + 1) * P, vis))));
                plan.part.push_back(plan.parts++);
            }
        }
    }
    return plan;
}

}  // namespace tvara
