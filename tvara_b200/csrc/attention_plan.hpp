// Host-side planning of a paged-attention launch: one work item per query
// row, or several (split-KV) for rows whose visible range is long relative to
// the batch, so that the grid covers every SM; split rows get a combine entry.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <vector>

namespace tvara {

struct AttnPlan {
    std::vector<int4> work;   // {row, table offset, pos begin, pos end}
    std::vector<int> part;    // partial slot or -1
    std::vector<int4> comb;   // {row, first part, parts, 0}
    int parts = 0;
};

inline AttnPlan plan_attention(const std::vector<int>& visible, const std::vector<int>& table_off, int tpb, int kv_heads,
                               std::size_t parts_cap, int sms = 148) {
    long long total = 0;
    for (int v : visible) total += v;
    const long long target = std::max<long long>(1, (long long)sms * 8 / std::max(1, kv_heads));
    long long P = std::max<long long>((long long)tpb * 8, (total + target - 1) / target);
    P = (P + tpb - 1) / tpb * tpb;
    auto count = [&](long long p) {
        long long n = 0;
        for (int v : visible)
            if (v > p) n += (v + p - 1) / p;
        return n;
    };
    while (count(P) > (long long)parts_cap) P *= 2;
    AttnPlan plan;
    for (std::size_t t = 0; t < visible.size(); ++t) {
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
