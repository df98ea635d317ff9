// C entry points over the reference engine's own headers -- TEST
// INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file against the Tvara
// source tree (core/include) into oracle/_ref/libtvara_refshim.so.  Tests
// use it to pin the C restatement in oracle/oracle.c, bench.py uses it as
// the reference CPU baseline.  No shipped code links it.
#include "tvara/attention.hpp"
#include "tvara/kv.hpp"
#include "tvara/paged_model.hpp"
#include "tvara/radix.hpp"
#include "tvara/simd.hpp"
#include "tvara/thread_pool.hpp"

#include <cstring>
#include <memory>
#include <string>

using namespace tvara;

namespace {
thread_local std::string shim_error;
template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        shim_error = e.what();
        return -1;
    }
}
std::span<const std::byte> bytes_of(const void* p, std::size_t n) {
    return {static_cast<const std::byte*>(p), n};
}
}  // namespace

extern "C" {
const char* ref_error() { return shim_error.c_str(); }

float ref_half_to_float(std::uint16_t h) { return quant::half_to_float(h); }

int ref_q4k_scale_min(const std::uint8_t* scales12, std::size_t g, unsigned* scale, unsigned* min) {
    return guarded([&] {
        auto v = quant::q4k_scale_min(bytes_of(scales12, 12), g);
        *scale = v[0];
        *min = v[1];
    });
}

// quant.hpp dequantize_* and model.hpp tensor_floats for F32/F16.
int ref_dequantize(int type, const void* src, std::size_t nbytes, float* out, std::size_t count) {
    return guarded([&] {
        auto in = bytes_of(src, nbytes);
        std::span<float> o(out, count);
        if (type == 8) quant::dequantize_q8_0(in, o);
        else if (type == 2) quant::dequantize_q4_0(in, o);
        else if (type == 12) quant::dequantize_q4_k(in, o);
        else if (type == 1) { for (std::size_t i = 0; i < count; ++i) out[i] = quant::half_to_float(quant::u16(in, 2 * i)); }
        else if (type == 0) std::memcpy(out, src, count * 4);
        else throw std::invalid_argument("unsupported type");
    });
}

int ref_matvec_f32(const float* w, std::size_t rows, std::size_t cols, const float* x, float* out) {
    return guarded([&] {
        quant::matvec_f32({w, rows * cols}, rows, cols, {x, cols}, {out, rows});
    });
}

int ref_matvec_quant(int type, const void* w, std::size_t nbytes, std::size_t rows, std::size_t cols,
                     const float* x, float* out) {
    return guarded([&] {
        quant::matvec_quant(bytes_of(w, nbytes), rows, cols, static_cast<unsigned>(type), {x, cols}, {out, rows});
    });
}

// The reference's fastest CPU path for one packed projection: int8
// activations, KernelDispatch (AVX2 when present) per row, rows split over
// `threads` workers with ThreadPool/partition_rows.  `tokens` rows of x.
int ref_matmul_dispatch(int type, const void* w, std::size_t nbytes, std::size_t rows, std::size_t cols,
                        const float* x, std::size_t tokens, float* out, std::size_t threads) {
    return guarded([&] {
        std::size_t block = type == 12 ? 256 : 32, width = type == 12 ? 144 : type == 8 ? 34 : 18;
        const std::size_t stride = cols / block * width;
        if (nbytes != rows * stride) throw std::invalid_argument("storage mismatch");
        KernelDispatch dispatch(false);
        auto in = bytes_of(w, nbytes);
        static std::unique_ptr<ThreadPool> pool;
        if (!pool || pool->size() != threads) pool = std::make_unique<ThreadPool>(threads);
        for (std::size_t t = 0; t < tokens; ++t) {
            auto act = quant::quantize_activations({x + t * cols, cols});
            pool->execute([&](std::size_t index) {
                auto [begin, end] = partition_rows(rows, index, threads);
                for (std::size_t r = begin; r < end; ++r) {
                    auto row = in.subspan(r * stride, stride);
                    out[t * rows + r] = type == 12 ? dispatch.q4k(row, act) : type == 8 ? dispatch.q8(row, act) : dispatch.q4(row, act);
                }
            });
        }
    });
}

// The reference's served projection: dequantised F32 weights times F32
// activations (quant.hpp:163-169), rows split over `threads` workers.
int ref_matmul_f32_threads(const float* w, std::size_t rows, std::size_t cols, const float* x, std::size_t tokens,
                           float* out, std::size_t threads) {
    return guarded([&] {
        static std::unique_ptr<ThreadPool> pool;
        if (!pool || pool->size() != threads) pool = std::make_unique<ThreadPool>(threads);
        for (std::size_t t = 0; t < tokens; ++t)
            pool->execute([&](std::size_t index) {
                auto [begin, end] = partition_rows(rows, index, threads);
                for (std::size_t r = begin; r < end; ++r)
                    out[t * rows + r] = quant::dot_f32({w + r * cols, cols}, {x + t * cols, cols});
            });
    });
}

int ref_rms_norm(const float* x, const float* w, std::size_t n, float eps, float* out) {
    return guarded([&] {
        auto v = rms_norm({x, n}, {w, n}, eps);
        std::copy(v.begin(), v.end(), out);
    });
}

int ref_rotary(float* x, std::size_t heads, std::size_t dim, std::size_t position, float theta, int interleaved) {
    return guarded([&] { rotary({x, heads * dim}, heads, dim, position, theta, interleaved != 0); });
}

// ---- paged cache (kv.hpp) ------------------------------------------------
struct ref_cache {
    PagedCache cache;
    std::unique_ptr<RadixCache> radix;
    explicit ref_cache(CacheGeometry g) : cache(g) {}
};

ref_cache* ref_cache_new(std::size_t layers, std::size_t kv_heads, std::size_t head_dim, std::size_t tpb,
                         std::size_t max_blocks) {
    try {
        return new ref_cache(CacheGeometry{layers, kv_heads, head_dim, tpb, max_blocks});
    } catch (const std::exception& e) {
        shim_error = e.what();
        return nullptr;
    }
}
void ref_cache_free(ref_cache* c) { delete c; }
std::uint64_t ref_cache_create(ref_cache* c) { return c->cache.create_sequence(); }
// Returns 0, -1 on error, -2 on CacheExhausted.
int ref_cache_append(ref_cache* c, std::uint64_t s, const float* keys, const float* values) {
    const auto n = c->cache.geometry().layers * c->cache.geometry().kv_width();
    try {
        c->cache.append(s, {keys, n}, {values, n});
        return 0;
    } catch (const CacheExhausted& e) {
        shim_error = e.what();
        return -2;
    } catch (const std::exception& e) {
        shim_error = e.what();
        return -1;
    }
}
int ref_cache_drop(ref_cache* c, std::uint64_t s) { return guarded([&] { c->cache.drop(s); }); }
std::uint64_t ref_cache_fork(ref_cache* c, std::uint64_t s) {
    std::uint64_t id = 0;
    guarded([&] { id = c->cache.fork(s); });
    return id;
}
int ref_cache_truncate(ref_cache* c, std::uint64_t s, std::size_t n) { return guarded([&] { c->cache.truncate(s, n); }); }
std::uint64_t ref_cache_import(ref_cache* c, std::uint64_t s, std::size_t n) {
    std::uint64_t id = 0;
    guarded([&] { id = c->cache.import_sequence(c->cache.sequence(s), n); });
    return id;
}
std::size_t ref_cache_available(ref_cache* c) { return c->cache.pool().available(); }
std::size_t ref_cache_references(ref_cache* c, std::size_t id) { return c->cache.pool().references_by_id(id); }
std::size_t ref_cache_length(ref_cache* c, std::uint64_t s) {
    std::size_t n = 0;
    guarded([&] { n = c->cache.sequence(s).length; });
    return n;
}
std::size_t ref_cache_table(ref_cache* c, std::uint64_t s, std::size_t* ids, std::uint64_t* gens) {
    std::size_t n = 0;
    guarded([&] {
        const auto& t = c->cache.sequence(s);
        for (auto b : t.blocks) { ids[n] = b.id; gens[n] = b.generation; ++n; }
    });
    return n;
}
int ref_cache_audit(ref_cache* c) {
    return guarded([&] {
        if (c->radix) c->cache.audit(c->radix->external_references());
        else c->cache.audit();
    });
}
float* ref_cache_block(ref_cache* c, std::uint64_t s, std::size_t position) {
    try {
        auto h = c->cache.physical_block(s, position);
        return c->cache.pool().data(h).data();
    } catch (const std::exception& e) {
        shim_error = e.what();
        return nullptr;
    }
}

// attention.hpp fused_paged_attention on this cache.
int ref_paged_attention(ref_cache* c, std::uint64_t s, std::size_t layer, std::size_t heads, const float* q,
                        const float* tail_k, const float* tail_v, std::size_t visible, float* out) {
    return guarded([&] {
        const auto& g = c->cache.geometry();
        ModelConfig cfg{16, heads * g.head_dim, 16, g.layers, heads, g.kv_heads, 1000000};
        const auto w = g.kv_width();
        auto v = fused_paged_attention({q, heads * g.head_dim}, c->cache, s, layer, cfg,
                                       tail_k ? std::span<const float>(tail_k, w) : std::span<const float>{},
                                       tail_v ? std::span<const float>(tail_v, w) : std::span<const float>{},
                                       visible ? visible : std::numeric_limits<std::size_t>::max());
        std::copy(v.begin(), v.end(), out);
    });
}

// ---- radix prefix cache (radix.hpp) -------------------------------------
int ref_radix_new(ref_cache* c, const char* isolation) {
    return guarded([&] { c->radix = std::make_unique<RadixCache>(c->cache, isolation); });
}
std::uint64_t ref_radix_insert(ref_cache* c, const std::int32_t* tokens, std::size_t n) {
    std::uint64_t id = 0;
    guarded([&] { id = c->radix->insert({tokens, n}); });
    return id;
}
std::size_t ref_radix_lookup(ref_cache* c, const std::int32_t* tokens, std::size_t n, std::uint64_t* node) {
    auto m = c->radix->lookup({tokens, n});
    *node = m.node;
    return m.tokens;
}
int ref_radix_attach(ref_cache* c, std::uint64_t node, std::uint64_t s) {
    return guarded([&] { c->radix->attach(node, s); });
}
std::uint64_t ref_radix_reuse(ref_cache* c, const std::int32_t* tokens, std::size_t n, int partial, std::size_t* length) {
    std::uint64_t id = 0;
    guarded([&] {
        auto r = c->radix->reuse({tokens, n}, partial != 0);
        id = r.first;
        *length = r.second;
    });
    return id;
}
int ref_radix_pin(ref_cache* c, std::uint64_t node) { return guarded([&] { c->radix->pin(node); }); }
int ref_radix_unpin(ref_cache* c, std::uint64_t node) { return guarded([&] { c->radix->unpin(node); }); }
int ref_radix_touch(ref_cache* c, std::uint64_t node) { return guarded([&] { c->radix->touch(node); }); }
int ref_radix_evict_one(ref_cache* c) {
    int r = 0;
    if (guarded([&] { r = c->radix->evict_one() ? 1 : 0; })) return -1;
    return r;
}
std::size_t ref_radix_size(ref_cache* c) { return c->radix->size(); }
}
