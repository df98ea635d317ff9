// Tensor-parallel shard of one rank: which query heads, KV heads and FFN rows
// it holds.  Q/K/V and gate/up are split by output rows (whole heads / FFN
// rows), o_proj and down_proj by input columns, so each rank's o_proj and
// down_proj produce a partial of the full hidden vector and one allreduce
// (sum) after each restores the residual on every rank.  Embedding, norms and
// the LM head are replicated.  The reference engine is single-device; this
// split has no counterpart there.
#pragma once

#include <stdexcept>
#include <string>

#include "common.hpp"
#include "gguf.hpp"

namespace tvara {

struct TpShard {
    int rank = 0, size = 1, head_dim = 0;
    int heads_begin = 0, heads = 0;        // query heads [heads_begin, heads_begin + heads)
    int kv_heads_begin = 0, kv_heads = 0;  // KV heads
    int ffn_begin = 0, ffn = 0;            // gate/up rows, down_proj columns
};

inline TpShard tp_shard(const gguf::File& f, const gguf::LlamaConfig& cfg, int rank, int size) {
    if (size < 1 || rank < 0 || rank >= size) throw std::invalid_argument("invalid tensor-parallel rank");
    if (cfg.heads % size || cfg.kv_heads % size || cfg.ffn % size)
        throw std::invalid_argument("tensor-parallel size must divide the head counts and FFN width");
    TpShard s;
    s.rank = rank;
    s.size = size;
    s.head_dim = int(cfg.head_dim());
    s.heads = int(cfg.heads) / size;
    s.kv_heads = int(cfg.kv_heads) / size;
    s.ffn = int(cfg.ffn) / size;
    s.heads_begin = rank * s.heads;
    s.kv_heads_begin = rank * s.kv_heads;
    s.ffn_begin = rank * s.ffn;
    if (s.heads / s.kv_heads > 8) throw std::invalid_argument("unsupported query/KV head ratio (1..8)");
    // column splits must fall on quantisation block boundaries
    auto check_cols = [&](const std::string& name, int cols) {
        std::size_t elems = 0, width = 0;
        if (!block_shape(static_cast<int>(f.info(name).type), elems, width))
            throw std::invalid_argument("unsupported native weight type");
        if (std::size_t(cols) % elems) throw std::invalid_argument("tensor-parallel split is not a whole number of blocks");
    };
    if (size > 1)
        for (std::size_t l = 0; l < cfg.layers; ++l) {
            const auto p = "blk." + std::to_string(l) + ".";
            check_cols(p + "attn_output.weight", s.heads * s.head_dim);
            check_cols(p + "ffn_down.weight", s.ffn);
        }
    return s;
}

}  // namespace tvara
