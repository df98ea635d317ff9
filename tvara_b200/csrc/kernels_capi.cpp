// Kernel-level C ABI (include/tvara_kernels.h): single hot-path kernels on
// caller-owned device memory.
#include "../../include/tvara_kernels.h"

#include <cstddef>
#include <cstring>
#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "attention_plan.hpp"
#include "kernels.cuh"

namespace tvara {
std::string& last_error();
}

namespace {

template <class F>
int guarded(F&& body) {
    tvara::last_error().clear();
    try {
        body();
        return 0;
    } catch (const std::exception& e) {
        tvara::last_error() = e.what();
        return -1;
    }
}

std::size_t align256(std::size_t n) { return (n + 255) & ~std::size_t(255); }

// Q4_K rows the tensor-core path reads packed (with side arrays).
bool has_q4k_side(int type, std::size_t cols) { return type == tvara::kQ4_K && cols % 256 == 0 && cols > 0; }

tvara::DeviceMatrix packed_view(int type, const void* packed, std::size_t rows, std::size_t cols) {
    std::size_t e = 0, w = 0;
    if (!tvara::block_shape(type, e, w)) throw std::invalid_argument("unsupported quantized type");
    if (!rows || !cols || cols % e || rows > 0x7fffffff || cols > 0x7fffffff)
        throw std::invalid_argument("invalid quantized matrix dimensions");
    if (type == tvara::kF32 && cols % 4) throw std::invalid_argument("F32 rows must be a multiple of 4 wide");
    if (type == tvara::kF16 && cols % 8) throw std::invalid_argument("F16 rows must be a multiple of 8 wide");
    tvara::DeviceMatrix m;
    m.type = type;
    m.rows = int(rows);
    m.cols = int(cols);
    m.qs_row = tvara::qs_row_bytes(type, cols);
    m.meta_row = tvara::meta_row_bytes(type, cols);
    m.qs = static_cast<const std::uint8_t*>(packed);
    m.meta = m.qs + align256(m.qs_row * rows);
    m.row_shift = reinterpret_cast<const signed char*>(m.meta + align256(m.meta_row * rows));
    if (has_q4k_side(type, cols)) {  // side arrays of the packed Q4_K tensor-core form, as launch_q4k_packed_form lays them
        const std::uint8_t* at = reinterpret_cast<const std::uint8_t*>(m.row_shift) + align256(rows);
        const std::size_t units = rows * (cols / 32);
        m.qsc = at;
        at += align256(units);
        m.qmin_hi = reinterpret_cast<const std::uint16_t*>(at);
        at += align256(units * 2);
        m.qmin_lo = reinterpret_cast<const std::uint16_t*>(at);
        at += align256(units * 2);
        m.qscale = reinterpret_cast<const float*>(at);
        at += align256(rows * (cols / 256) * 4);
        m.qmin_shift = reinterpret_cast<const signed char*>(at);
    }
    return m;
}

struct AttnLayout {
    tvara::AttnPlan plan;
    std::size_t off_tables = 0, off_work = 0, off_chunk = 0, off_part = 0, off_comb = 0, off_partial = 0, off_err = 0,
                total = 0;
};

constexpr std::size_t kPartsCap = 16384;

AttnLayout layout_for(const tvara_attention_args* a) {
    // kv_scales was appended: the shorter struct stays valid for F32 / F16 pools
    if (!a || a->struct_size < offsetof(tvara_attention_args, kv_scales))
        throw std::invalid_argument("invalid attention arguments");
    if (a->kv_dtype > TVARA_KV_I8 ||
        (a->kv_dtype == TVARA_KV_I8 &&
         (a->struct_size < offsetof(tvara_attention_args, kv_scales) + sizeof(a->kv_scales) || !a->kv_scales)))
        throw std::invalid_argument("invalid KV dtype or missing int8 scales");
    if (!a->heads || !a->kv_heads || a->heads % a->kv_heads || !a->block_tokens || !a->layers || a->layer >= a->layers)
        throw std::invalid_argument("invalid attention geometry");
    AttnLayout L;
    std::vector<int> vis(a->n_queries), off(a->n_queries);
    if (a->n_queries && (!a->visible || !a->table_offset || !a->tables))
        throw std::invalid_argument("invalid attention arguments");
    if (!a->max_blocks || a->max_blocks > 0x7fffffff) throw std::invalid_argument("invalid KV pool size");
    for (std::size_t i = 0; i < a->n_queries; ++i) {
        if (!a->visible[i]) throw std::invalid_argument("empty fused attention");
        const std::size_t blocks = (a->visible[i] + a->block_tokens - 1) / a->block_tokens;
        if (a->table_offset[i] + blocks > a->tables_len) throw std::invalid_argument("block table shorter than visible range");
        // every block a query reads must be a pool block: checked here, before
        // anything is enqueued, rather than left to the kernels' guard
        for (std::size_t b = 0; b < blocks; ++b) {
            const std::int32_t id = a->tables[a->table_offset[i] + b];
            if (id < 0 || std::size_t(id) >= a->max_blocks) throw std::invalid_argument("block id outside the KV pool");
        }
        vis[i] = int(a->visible[i]);
        off[i] = int(a->table_offset[i]);
    }
    L.plan = tvara::plan_attention(
        vis, off, int(a->block_tokens), int(a->kv_heads), kPartsCap, 148,
        tvara::attention_chunk_rows(int(a->kv_dtype), int(a->head_dim), int(a->heads / a->kv_heads),
                                    int(a->block_tokens)));
    std::size_t at = 0;
    L.off_tables = at;
    at = align256(at + a->tables_len * 4);
    L.off_work = at;
    at = align256(at + L.plan.work.size() * 16);
    L.off_chunk = at;
    at = align256(at + L.plan.chunk.size() * 16);
    L.off_part = at;
    at = align256(at + L.plan.part.size() * 4);
    L.off_comb = at;
    at = align256(at + L.plan.comb.size() * 16);
    L.off_partial = at;
    at = align256(at + std::size_t(L.plan.parts) * a->heads * (a->head_dim + 2) * 4);
    L.off_err = at;
    L.total = align256(at + 4);
    return L;
}

}  // namespace

extern "C" {

int tvara_dequantize(int type, const void* blocks, size_t nblocks, float* out, void* stream) {
    return guarded([&] { tvara::launch_dequantize(type, blocks, nblocks, out, static_cast<cudaStream_t>(stream)); });
}

size_t tvara_packed_bytes(int type, size_t rows, size_t cols) {
    std::size_t e = 0, w = 0;
    if (!tvara::block_shape(type, e, w) || !cols || cols % e) return 0;
    return align256(tvara::qs_row_bytes(type, cols) * rows) + align256(tvara::meta_row_bytes(type, cols) * rows) +
           align256(rows) + (has_q4k_side(type, cols) ? tvara::q4k_packed_form_bytes(int(rows), int(cols)) : 0);
}

int tvara_pack(int type, const void* gguf_rows, size_t rows, size_t cols, void* packed, void* stream) {
    return guarded([&] {
        auto m = packed_view(type, packed, rows, cols);
        auto s = static_cast<cudaStream_t>(stream);
        tvara::launch_repack(type, gguf_rows, int(rows), int(cols), const_cast<std::uint8_t*>(m.qs),
                             const_cast<std::uint8_t*>(m.meta), s);
        tvara::launch_row_shift(m, const_cast<signed char*>(m.row_shift), s);
        if (has_q4k_side(type, cols)) {
            tvara::DeviceMatrix side = m;
            tvara::launch_q4k_packed_form(side, const_cast<signed char*>(m.row_shift) + align256(rows), s);
        }
    });
}

namespace {
std::size_t pow2_at_least(std::size_t n) {
    std::size_t p = 1;
    while (p < n) p <<= 1;
    return p;
}
}  // namespace

size_t tvara_sample_workspace(size_t rows, size_t max_history) {
    if (!rows || max_history > 16384) return 0;
    return rows * (8 + 4 + 24) + rows * pow2_at_least(std::max<std::size_t>(max_history, 1)) * 8 + 256;
}

int tvara_sample_logits(const float* logits, size_t rows, size_t vocab, const int32_t* history,
                        const uint64_t* history_offsets, const double* repetition, const double* frequency,
                        const double* presence, const uint32_t* allowed, uint32_t top_k, uint32_t* argmax,
                        int32_t* status, double* top_values, uint32_t* top_ids, void* workspace,
                        size_t workspace_bytes, void* stream) {
    return guarded([&] {
        if (!logits || !rows || !vocab || vocab > 0x7fffffff || rows > 0x7fffffff || !history_offsets || !argmax ||
            !status || !workspace)
            throw std::invalid_argument("invalid sampling arguments");
        if (top_k > 64 || top_k > vocab) throw std::invalid_argument("top-k candidates must be between 0 and 64");
        if (top_k && (!top_values || !top_ids)) throw std::invalid_argument("invalid top-k output buffers");
        std::vector<long long> hoff(rows);
        std::vector<int> hlen(rows);
        std::vector<double> par(rows * 3);
        std::size_t longest = 0;
        for (std::size_t r = 0; r < rows; ++r) {
            if (history_offsets[r + 1] < history_offsets[r]) throw std::invalid_argument("invalid history offsets");
            const std::size_t n = history_offsets[r + 1] - history_offsets[r];
            if (n > 16384) throw std::invalid_argument("device sampling holds at most 16384 tokens of history");
            if (n && !history) throw std::invalid_argument("invalid sampling arguments");
            hoff[r] = (long long)history_offsets[r];
            hlen[r] = int(n);
            longest = std::max(longest, n);
            par[3 * r] = repetition ? repetition[r] : 1.0;
            par[3 * r + 1] = frequency ? frequency[r] : 0.0;
            par[3 * r + 2] = presence ? presence[r] : 0.0;
            if (!std::isfinite(par[3 * r]) || par[3 * r] <= 0 || !std::isfinite(par[3 * r + 1]) ||
                !std::isfinite(par[3 * r + 2]))
                throw std::invalid_argument("Invalid sampling filters or penalties");
        }
        if (workspace_bytes < tvara_sample_workspace(rows, longest))
            throw std::invalid_argument("sampling workspace too small");
        const std::size_t cap = pow2_at_least(std::max<std::size_t>(longest, 1));
        auto* base = static_cast<unsigned char*>(workspace);
        auto s = static_cast<cudaStream_t>(stream);
        // [pen rows x cap doubles][params rows x 3 doubles][hoff rows][hlen rows]
        double* pen = reinterpret_cast<double*>(base);
        double* d_par = pen + rows * cap;
        long long* d_hoff = reinterpret_cast<long long*>(d_par + rows * 3);
        int* d_hlen = reinterpret_cast<int*>(d_hoff + rows);
        TVARA_CUDA(cudaMemcpyAsync(d_par, par.data(), par.size() * 8, cudaMemcpyHostToDevice, s));
        TVARA_CUDA(cudaMemcpyAsync(d_hoff, hoff.data(), hoff.size() * 8, cudaMemcpyHostToDevice, s));
        TVARA_CUDA(cudaMemcpyAsync(d_hlen, hlen.data(), hlen.size() * 4, cudaMemcpyHostToDevice, s));
        tvara::SampleJob j;
        j.logits = logits;
        j.ld = (long long)vocab;
        j.rows = int(rows);
        j.vocab = int(vocab);
        j.hist = history;
        j.hoff = d_hoff;
        j.hlen = d_hlen;
        j.hist_cap = int(cap);
        j.params = d_par;
        j.allowed = allowed;
        j.words = int((vocab + 31) / 32);
        j.top_k = int(top_k);
        j.pen = pen;
        j.pen_stride = (long long)cap;
        j.argmax = argmax;
        j.status = status;
        j.top_val = top_values;
        j.top_id = top_ids;
        tvara::launch_sample(j, s);
    });
}

int tvara_kv_quantize(const float* rows, size_t n, size_t dim, int8_t* codes, float* scales, void* stream) {
    return guarded([&] {
        if (!rows || !codes || !scales || !n || !dim || n > 0x7fffffff || dim > 0x7fffffff)
            throw std::invalid_argument("invalid KV quantize arguments");
        auto s = static_cast<cudaStream_t>(stream);
        int* err = nullptr;
        TVARA_CUDA(cudaMallocAsync(&err, sizeof(int), s));
        TVARA_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
        tvara::launch_kv_quantize(rows, int(n), int(dim), reinterpret_cast<signed char*>(codes), scales, err, s);
        int host = 0;
        TVARA_CUDA(cudaMemcpyAsync(&host, err, sizeof(int), cudaMemcpyDeviceToHost, s));
        TVARA_CUDA(cudaFreeAsync(err, s));
        TVARA_CUDA(cudaStreamSynchronize(s));
        if (host) throw std::invalid_argument("Nonfinite KV input");
    });
}

size_t tvara_quant_matmul_workspace(size_t cols, size_t tokens) {
    return tokens <= 4 ? 0 : tvara::gemm_tc_workspace(int(tokens), int(cols));
}

int tvara_quant_matmul(int type, const void* packed, size_t rows, size_t cols, const float* x, size_t tokens,
                       float* y, void* workspace, size_t workspace_bytes, void* stream) {
    return guarded([&] {
        tvara::GemmArgs g;
        g.w = packed_view(type, packed, rows, cols);
        g.x = x;
        g.ldx = int(cols);
        g.tokens = int(tokens);
        g.y = y;
        g.ldy = int(rows);
        g.epilogue = tvara::kStore;
        if (tokens > 4 && workspace_bytes < tvara::gemm_tc_workspace(int(tokens), int(cols)))
            throw std::invalid_argument("matmul workspace too small");
        tvara::launch_projection(g, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
    });
}

size_t tvara_paged_attention_workspace(const tvara_attention_args* a) {
    std::size_t n = 0;
    if (guarded([&] { n = layout_for(a).total; })) return 0;
    return n;
}

int tvara_paged_attention(const tvara_attention_args* a, void* workspace, size_t workspace_bytes, void* stream) {
    return guarded([&] {
        auto L = layout_for(a);
        if (!workspace || workspace_bytes < L.total) throw std::invalid_argument("attention workspace too small");
        auto s = static_cast<cudaStream_t>(stream);
        // The call stages its tables from a host buffer that dies on return and
        // waits for the kernels' error word: it cannot be recorded into a graph.
        cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
        TVARA_CUDA(cudaStreamIsCapturing(s, &capturing));
        if (capturing != cudaStreamCaptureStatusNone)
            throw std::invalid_argument("paged attention cannot be captured into a CUDA graph");
        auto* base = static_cast<std::uint8_t*>(workspace);
        std::vector<std::uint8_t> host(L.off_partial);
        std::memcpy(host.data() + L.off_tables, a->tables, a->tables_len * 4);
        std::memcpy(host.data() + L.off_work, L.plan.work.data(), L.plan.work.size() * 16);
        std::memcpy(host.data() + L.off_chunk, L.plan.chunk.data(), L.plan.chunk.size() * 16);
        std::memcpy(host.data() + L.off_part, L.plan.part.data(), L.plan.part.size() * 4);
        std::memcpy(host.data() + L.off_comb, L.plan.comb.data(), L.plan.comb.size() * 16);
        TVARA_CUDA(cudaMemcpyAsync(base, host.data(), host.size(), cudaMemcpyHostToDevice, s));
        TVARA_CUDA(cudaMemsetAsync(base + L.off_err, 0, 4, s));
        tvara::AttnArgs g;
        g.q = a->q;
        g.out = a->out;
        g.kv = a->pool;
        g.kv_f16 = a->kv_dtype == TVARA_KV_F16;
        g.kv_i8 = a->kv_dtype == TVARA_KV_I8;
        g.kv_scales = g.kv_i8 ? a->kv_scales : nullptr;
        g.hq = int(a->heads);
        g.hkv = int(a->kv_heads);
        g.dim = int(a->head_dim);
        g.tpb = int(a->block_tokens);
        g.kind_stride = (long long)a->kv_heads * a->block_tokens * a->head_dim;
        g.layer_offset = (long long)a->layer * 2 * g.kind_stride;
        g.block_stride = (long long)a->layers * 2 * g.kind_stride;
        g.tables = reinterpret_cast<const int*>(base + L.off_tables);
        g.work = reinterpret_cast<const int4*>(base + L.off_work);
        g.work_part = reinterpret_cast<const int*>(base + L.off_part);
        g.n_work = int(L.plan.work.size());
        g.partial = reinterpret_cast<float*>(base + L.off_partial);
        g.combine = reinterpret_cast<const int4*>(base + L.off_comb);
        g.n_combine = int(L.plan.comb.size());
        g.max_blocks = int(a->max_blocks);
        g.chunk_work = reinterpret_cast<const int4*>(base + L.off_chunk);
        g.n_chunk = int(L.plan.chunk.size());
        g.err = reinterpret_cast<int*>(base + L.off_err);
        tvara::launch_attention(g, s);
        // the kernels' error word: 2 a block id outside the pool, 4 a bounded
        // wait on a copy that never completed
        int word = 0;
        TVARA_CUDA(cudaMemcpyAsync(&word, base + L.off_err, sizeof(int), cudaMemcpyDeviceToHost, s));
        TVARA_CUDA(cudaStreamSynchronize(s));
        if (word == 2) throw std::runtime_error("paged attention read a block id outside the KV pool");
        if (word) throw std::runtime_error("paged attention timed out waiting for a KV copy (error " +
                                           std::to_string(word) + ")");
    });
}

}  // extern "C"
