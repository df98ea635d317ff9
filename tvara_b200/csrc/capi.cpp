// C ABI of the engine (include/tvara_capi.h).  The first eleven entry points
// keep the reference's contract (core/src/c_api.cpp:38-78): each clears the
// thread's error string, catches every exception into it, and serialises
// work on a handle with one mutex.
#include "../../include/tvara_capi.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstddef>
#include <cstring>
#include <limits>
#include <memory>
#include <mutex>
#include <string>

#include "engine.hpp"
#include "gguf.hpp"
#include "tp_plan.hpp"

struct tvara_model {
    std::unique_ptr<tvara::Engine> engine;
    std::mutex mutex;
};

struct tvara_kv_book {
    tvara::SequenceBook book;
    std::unique_ptr<tvara::PrefixTrie> trie;  // declared after book: released first
    explicit tvara_kv_book(tvara::CacheGeometry g) : book(g) {}
    tvara::PrefixTrie& prefixes() {
        if (!trie) trie = std::make_unique<tvara::PrefixTrie>(book, "tvara-kv-book");
        return *trie;
    }
};

#include <atomic>

namespace tvara {
std::string& last_error() {
    thread_local std::string message;
    return message;
}
namespace {
std::atomic<unsigned long long> g_launches{0};
}
void note_launches(unsigned long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
unsigned long long launches() { return g_launches.load(std::memory_order_relaxed); }
}  // namespace tvara

// The calling thread's message (evaluated per use: the string is thread-local).
#define error_message (::tvara::last_error())

namespace {

template <class R, class F>
R guarded(R fail, F&& body) {
    error_message.clear();
    try {
        return body();
    } catch (const std::exception& e) {
        error_message = e.what();
        return fail;
    } catch (...) {
        error_message = "unknown native error";
        return fail;
    }
}

tvara::Engine& engine_of(tvara_model* m) {
    if (!m || !m->engine) throw std::invalid_argument("closed model");
    TVARA_CUDA(cudaSetDevice(m->engine->device()));
    return *m->engine;
}

tvara_model* open_model(const char* path, size_t blocks, size_t tokens, const tvara_open_options* o) {
    if (!path || !*path) throw std::invalid_argument("empty model path");
    tvara::EngineOptions opt;
    if (o) {
        // the struct grows at its end; weight_planes is the first optional member
        if (o->struct_size < offsetof(tvara_open_options, weight_planes))
            throw std::invalid_argument("invalid open options size");
        opt.device = o->device;
        if (o->kv_dtype > TVARA_KV_I8) throw std::invalid_argument("invalid KV dtype");
        opt.kv_f16 = o->kv_dtype == TVARA_KV_F16;
        opt.kv_i8 = o->kv_dtype == TVARA_KV_I8;
        if (o->max_step_tokens) opt.max_step_tokens = int(o->max_step_tokens);
        opt.tp_rank = int(o->tp_rank);
        opt.tp_size = o->tp_size ? int(o->tp_size) : 1;
        if (o->nccl_id) {
            std::memcpy(opt.nccl_id.data(), o->nccl_id, opt.nccl_id.size());
            opt.has_nccl_id = true;
        }
        if (o->struct_size >= offsetof(tvara_open_options, weight_planes) + sizeof(uint32_t)) {
            if (o->weight_planes > 4) throw std::invalid_argument("invalid weight planes option");
            opt.weight_planes = int(o->weight_planes);
        }
    }
    auto m = std::make_unique<tvara_model>();
    m->engine = std::make_unique<tvara::Engine>(path, blocks, tokens, opt);
    return m.release();
}
}  // namespace

extern "C" {

tvara_model* tvara_model_open(const char* path, size_t max_blocks, size_t block_tokens) {
    return guarded<tvara_model*>(nullptr, [&] { return open_model(path, max_blocks, block_tokens, nullptr); });
}

tvara_model* tvara_model_open_ex(const char* path, size_t max_blocks, size_t block_tokens,
                                 const tvara_open_options* options) {
    return guarded<tvara_model*>(nullptr, [&] { return open_model(path, max_blocks, block_tokens, options); });
}

int tvara_model_weight_bytes(tvara_model* model, size_t* packed, size_t* planes) {
    return guarded<int>(-1, [&] {
        if (!model || !model->engine) throw std::invalid_argument("closed model");
        if (packed) *packed = model->engine->weight_bytes();
        if (planes) *planes = model->engine->plane_bytes();
        return 0;
    });
}

int tvara_tp_shard(const char* path, uint32_t tp_rank, uint32_t tp_size, tvara_tp_shard_info* out) {
    return guarded<int>(-1, [&] {
        if (!path || !*path) throw std::invalid_argument("empty model path");
        if (!out || out->struct_size < sizeof(tvara_tp_shard_info)) throw std::invalid_argument("invalid shard output");
        tvara::gguf::File f(path);
        const auto cfg = tvara::gguf::llama_config(f.doc());
        tvara::gguf::validate_llama_tensors(f.doc(), cfg);
        const auto s = tvara::tp_shard(f, cfg, int(tp_rank), tp_size ? int(tp_size) : 1);
        out->head_dim = uint32_t(s.head_dim);
        out->heads_begin = uint32_t(s.heads_begin);
        out->heads = uint32_t(s.heads);
        out->kv_heads_begin = uint32_t(s.kv_heads_begin);
        out->kv_heads = uint32_t(s.kv_heads);
        out->ffn_begin = uint32_t(s.ffn_begin);
        out->ffn = uint32_t(s.ffn);
        return 0;
    });
}

void tvara_model_close(tvara_model* model) {
    if (model && model->engine) cudaSetDevice(model->engine->device());
    delete model;
}

size_t tvara_model_vocab_size(tvara_model* model) {
    if (!model) {
        error_message = "closed model";
        return 0;
    }
    return model->engine->config().vocab;
}

size_t tvara_model_context_size(tvara_model* model) {
    if (!model) {
        error_message = "closed model";
        return 0;
    }
    return model->engine->config().context;
}

const char* tvara_last_error(void) { return error_message.c_str(); }

const char* tvara_model_metadata(tvara_model* model) {
    if (!model) {
        error_message = "closed model";
        return nullptr;
    }
    return model->engine->metadata().c_str();
}

uint64_t tvara_sequence_create(tvara_model* model) {
    return guarded<uint64_t>(0, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        return e.book().create_sequence();
    });
}

int tvara_sequence_decode(tvara_model* model, uint64_t sequence, uint32_t token, float* logits, size_t count) {
    return guarded<int>(-1, [&] {
        if (!model || !logits || count != model->engine->config().vocab)
            throw std::invalid_argument("invalid logit output buffer");
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        const uint32_t cu[2] = {0, 1};
        e.step({&sequence, 1}, {cu, 2}, {&token, 1}, false, logits, nullptr);
        return 0;
    });
}

int tvara_sequence_drop(tvara_model* model, uint64_t sequence) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        e.book().drop(sequence);
        return 0;
    });
}

int tvara_sequence_decode_batch(tvara_model* model, uint64_t sequence, const uint32_t* tokens, size_t token_count,
                                float* logits, size_t count) {
    return guarded<int>(-1, [&] {
        if (!model || (!tokens && token_count) || (!logits && count)) throw std::invalid_argument("invalid batch buffers");
        const auto vocab = model->engine->config().vocab;
        if (token_count > std::numeric_limits<size_t>::max() / vocab || count != token_count * vocab)
            throw std::invalid_argument("invalid batch dimensions");
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        const auto length = e.book().sequence(sequence).length;
        if (token_count > e.config().context - length) throw std::invalid_argument("batch exceeds context");
        for (size_t i = 0; i < token_count; ++i)
            if (tokens[i] >= vocab) throw std::invalid_argument("invalid batch token");
        if (!token_count) return 0;
        const uint32_t cu[2] = {0, uint32_t(token_count)};
        e.step({&sequence, 1}, {cu, 2}, {tokens, token_count}, true, logits, nullptr);
        return 0;
    });
}

int tvara_sequence_truncate(tvara_model* model, uint64_t sequence, size_t length) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        e.book().truncate(sequence, length);
        return 0;
    });
}

int tvara_batch_step(tvara_model* model, size_t n_seq, const uint64_t* sequences, const uint32_t* cu_tokens,
                     const uint32_t* tokens, uint32_t flags, float* logits, size_t count, uint32_t* argmax,
                     size_t argmax_count) {
    return guarded<int>(-1, [&] {
        if (!model || !n_seq || !sequences || !cu_tokens || !tokens) throw std::invalid_argument("invalid batch buffers");
        if (flags & ~uint32_t(TVARA_STEP_ALL_LOGITS | TVARA_STEP_FINITE_ARGMAX))
            throw std::invalid_argument("unknown step flags");
        const size_t total = cu_tokens[n_seq];
        const bool all = flags & TVARA_STEP_ALL_LOGITS;
        const size_t rows = all ? total : n_seq;
        const auto vocab = model->engine->config().vocab;
        if (rows > std::numeric_limits<size_t>::max() / vocab) throw std::invalid_argument("invalid batch dimensions");
        if (logits && count != rows * vocab) throw std::invalid_argument("invalid logit output buffer");
        if (argmax && argmax_count != rows) throw std::invalid_argument("invalid argmax output buffer");
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        e.step({sequences, n_seq}, {cu_tokens, n_seq + 1}, {tokens, total}, all, logits, argmax,
               (flags & TVARA_STEP_FINITE_ARGMAX) != 0);
        return 0;
    });
}

int tvara_batch_sample(tvara_model* model, size_t n_seq, const uint64_t* sequences, const uint32_t* cu_tokens,
                       const uint32_t* tokens, const tvara_sampling* sampling, float* logits, size_t count,
                       uint32_t* argmax, int32_t* status, double* top_values, uint32_t* top_ids) {
    return guarded<int>(-1, [&] {
        if (!model || !n_seq || !sequences || !cu_tokens || !tokens) throw std::invalid_argument("invalid batch buffers");
        if (!sampling || sampling->struct_size < sizeof(tvara_sampling))
            throw std::invalid_argument("invalid sampling arguments");
        if (sampling->top_k > tvara::kSampleMaxK) throw std::invalid_argument("top-k candidates must be between 0 and 64");
        if (sampling->top_k && (!top_values || !top_ids)) throw std::invalid_argument("invalid top-k output buffers");
        for (size_t i = 0; i < n_seq; ++i) {
            const double r = sampling->repetition ? sampling->repetition[i] : 1.0;
            const double f = sampling->frequency ? sampling->frequency[i] : 0.0;
            const double p = sampling->presence ? sampling->presence[i] : 0.0;
            if (!std::isfinite(r) || r <= 0 || !std::isfinite(f) || !std::isfinite(p))
                throw std::invalid_argument("Invalid sampling filters or penalties");
        }
        const size_t total = cu_tokens[n_seq];
        if (logits && (n_seq > std::numeric_limits<size_t>::max() / model->engine->config().vocab ||
                       count != n_seq * model->engine->config().vocab))
            throw std::invalid_argument("invalid logit output buffer");
        tvara::SampleSpec spec;
        spec.repetition = sampling->repetition;
        spec.frequency = sampling->frequency;
        spec.presence = sampling->presence;
        spec.allowed = sampling->allowed;
        spec.top_k = int(sampling->top_k);
        spec.argmax = argmax;
        spec.status = status;
        spec.top_values = top_values;
        spec.top_ids = top_ids;
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        e.step({sequences, n_seq}, {cu_tokens, n_seq + 1}, {tokens, total}, false, logits, nullptr, false, &spec);
        return 0;
    });
}

uint64_t tvara_sequence_fork(tvara_model* model, uint64_t sequence) {
    return guarded<uint64_t>(0, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        return e.book().fork(sequence);
    });
}

int tvara_sequence_length(tvara_model* model, uint64_t sequence, size_t* length) {
    return guarded<int>(-1, [&] {
        if (!length) throw std::invalid_argument("invalid output pointer");
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        *length = e.book().sequence(sequence).length;
        return 0;
    });
}

int tvara_kv_stats(tvara_model* model, size_t* available, size_t* max_blocks) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        if (available) *available = e.book().ledger().available();
        if (max_blocks) *max_blocks = e.book().geometry().max_blocks;
        return 0;
    });
}

int tvara_kv_audit(tvara_model* model) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        const auto ext = e.radix().external_references();
        e.book().audit(ext);
        return 0;
    });
}

int tvara_sequence_blocks(tvara_model* model, uint64_t sequence, uint64_t* ids, uint64_t* generations,
                          size_t capacity, size_t* count) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        const auto& t = e.book().sequence(sequence);
        if (count) *count = t.blocks.size();
        for (size_t i = 0; i < t.blocks.size() && i < capacity; ++i) {
            if (ids) ids[i] = t.blocks[i].id;
            if (generations) generations[i] = t.blocks[i].generation;
        }
        return 0;
    });
}

int tvara_kv_references(tvara_model* model, size_t id, size_t* references) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        if (references) *references = e.book().ledger().references_by_id(id);
        return 0;
    });
}

int tvara_model_profile(tvara_model* model, int enable) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        e.set_profiling(enable != 0);
        return 0;
    });
}

int tvara_model_profile_read(tvara_model* model, double* ms, uint64_t* groups, size_t capacity) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        double t[tvara::Engine::kProfClasses];
        unsigned long long n[tvara::Engine::kProfClasses];
        e.profile_read(t, n);
        for (size_t i = 0; i < capacity && i < size_t(tvara::Engine::kProfClasses); ++i) {
            if (ms) ms[i] = t[i];
            if (groups) groups[i] = n[i];
        }
        return int(tvara::Engine::kProfClasses);
    });
}

uint64_t tvara_kernel_launches(void) { return tvara::launches(); }

int tvara_model_step_bytes(tvara_model* model, uint64_t* h2d, uint64_t* d2h) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        if (h2d) *h2d = e.last_h2d();
        if (d2h) *d2h = e.last_d2h();
        return 0;
    });
}

void* tvara_model_stream(tvara_model* model) {
    return guarded<void*>(nullptr, [&] { return static_cast<void*>(engine_of(model).stream()); });
}

int tvara_kv_pool(tvara_model* model, tvara_kv_pool_info* info) {
    return guarded<int>(-1, [&] {
        if (!info) throw std::invalid_argument("invalid output pointer");
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        const auto& g = e.book().geometry();
        info->base = e.kv_pool();
        info->max_blocks = g.max_blocks;
        info->block_elements = size_t(e.block_elements());
        info->kv_dtype = e.options().kv_i8 ? TVARA_KV_I8 : e.options().kv_f16 ? TVARA_KV_F16 : TVARA_KV_F32;
        info->layers = uint32_t(g.layers);
        info->kv_heads = uint32_t(e.local_kv_heads());
        info->head_dim = uint32_t(g.head_dim);
        info->block_tokens = uint32_t(g.tokens_per_block);
        return 0;
    });
}

int tvara_kv_pool_scales(tvara_model* model, float** scales) {
    return guarded<int>(-1, [&] {
        if (!scales) throw std::invalid_argument("invalid output pointer");
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        *scales = e.kv_scales();
        return 0;
    });
}

int tvara_sequence_reserve(tvara_model* model, uint64_t sequence, size_t count) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        e.reserve(sequence, count);
        return 0;
    });
}

uint64_t tvara_prefix_insert(tvara_model* model, const int32_t* tokens, size_t token_count, uint64_t sequence) {
    return guarded<uint64_t>(0, [&] {
        if (!tokens && token_count) throw std::invalid_argument("invalid token buffer");
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        const auto node = e.radix().insert({tokens, token_count});
        e.radix().attach(node, sequence);
        return node;
    });
}

uint64_t tvara_prefix_reuse(tvara_model* model, const int32_t* tokens, size_t token_count, int partial,
                            size_t* reused) {
    return guarded<uint64_t>(0, [&] {
        if (!tokens && token_count) throw std::invalid_argument("invalid token buffer");
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        auto r = e.radix().reuse({tokens, token_count}, partial != 0);
        if (reused) *reused = r.second;
        return r.first;
    });
}

int tvara_prefix_lookup(tvara_model* model, const int32_t* tokens, size_t token_count, uint64_t* node,
                        size_t* matched) {
    return guarded<int>(-1, [&] {
        if (!tokens && token_count) throw std::invalid_argument("invalid token buffer");
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        auto r = e.radix().lookup({tokens, token_count});
        if (node) *node = r.first;
        if (matched) *matched = r.second;
        return 0;
    });
}

int tvara_prefix_pin(tvara_model* model, uint64_t node) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        e.radix().pin(node);
        return 0;
    });
}

int tvara_prefix_unpin(tvara_model* model, uint64_t node) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        e.radix().unpin(node);
        return 0;
    });
}

int tvara_prefix_touch(tvara_model* model, uint64_t node) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        e.radix().touch(node);
        return 0;
    });
}

int tvara_prefix_evict_one(tvara_model* model) {
    return guarded<int>(-1, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        return e.radix().evict_one() ? 1 : 0;
    });
}

size_t tvara_prefix_size(tvara_model* model) {
    return guarded<size_t>(0, [&] {
        auto& e = engine_of(model);
        std::lock_guard lock(model->mutex);
        return e.radix().size();
    });
}

// ---- host-only accounting book ---------------------------------------------
tvara_kv_book* tvara_kv_book_new(size_t layers, size_t kv_heads, size_t head_dim, size_t block_tokens,
                                 size_t max_blocks) {
    return guarded<tvara_kv_book*>(nullptr, [&] {
        return new tvara_kv_book(tvara::CacheGeometry{layers, kv_heads, head_dim, block_tokens, max_blocks});
    });
}
void tvara_kv_book_free(tvara_kv_book* book) { delete book; }
uint64_t tvara_kv_book_create(tvara_kv_book* b) {
    return guarded<uint64_t>(0, [&] { return b->book.create_sequence(); });
}
int tvara_kv_book_append(tvara_kv_book* b, uint64_t s) {
    error_message.clear();
    try {
        b->book.append(s);
        return 0;
    } catch (const tvara::CacheExhausted& e) {
        error_message = e.what();
        return -2;
    } catch (const std::exception& e) {
        error_message = e.what();
        return -1;
    }
}
int tvara_kv_book_drop(tvara_kv_book* b, uint64_t s) {
    return guarded<int>(-1, [&] {
        b->book.drop(s);
        return 0;
    });
}
uint64_t tvara_kv_book_fork(tvara_kv_book* b, uint64_t s) {
    return guarded<uint64_t>(0, [&] { return b->book.fork(s); });
}
int tvara_kv_book_truncate(tvara_kv_book* b, uint64_t s, size_t n) {
    return guarded<int>(-1, [&] {
        b->book.truncate(s, n);
        return 0;
    });
}
uint64_t tvara_kv_book_import(tvara_kv_book* b, uint64_t s, size_t n) {
    return guarded<uint64_t>(0, [&] { return b->book.import_sequence(b->book.sequence(s), n); });
}
size_t tvara_kv_book_available(tvara_kv_book* b) { return b->book.ledger().available(); }
size_t tvara_kv_book_references(tvara_kv_book* b, size_t id) {
    return guarded<size_t>(0, [&] { return b->book.ledger().references_by_id(id); });
}
int tvara_kv_book_table(tvara_kv_book* b, uint64_t s, uint64_t* ids, uint64_t* gens, size_t capacity, size_t* count) {
    return guarded<int>(-1, [&] {
        const auto& t = b->book.sequence(s);
        if (count) *count = t.blocks.size();
        for (size_t i = 0; i < t.blocks.size() && i < capacity; ++i) {
            if (ids) ids[i] = t.blocks[i].id;
            if (gens) gens[i] = t.blocks[i].generation;
        }
        return 0;
    });
}
int tvara_kv_book_audit(tvara_kv_book* b) {
    return guarded<int>(-1, [&] {
        if (b->trie) {
            const auto held = b->trie->external_references();
            b->book.audit(held);
        } else {
            b->book.audit();
        }
        return 0;
    });
}
uint64_t tvara_kv_book_prefix_insert(tvara_kv_book* b, const int32_t* tokens, size_t token_count) {
    return guarded<uint64_t>(0, [&] {
        if (!tokens && token_count) throw std::invalid_argument("invalid token buffer");
        return b->prefixes().insert({tokens, token_count});
    });
}
int tvara_kv_book_prefix_attach(tvara_kv_book* b, uint64_t node, uint64_t sequence) {
    return guarded<int>(-1, [&] {
        b->prefixes().attach(node, sequence);
        return 0;
    });
}
int tvara_kv_book_prefix_lookup(tvara_kv_book* b, const int32_t* tokens, size_t token_count, uint64_t* node,
                                size_t* matched) {
    return guarded<int>(-1, [&] {
        if (!tokens && token_count) throw std::invalid_argument("invalid token buffer");
        const auto r = b->prefixes().lookup({tokens, token_count});
        if (node) *node = r.first;
        if (matched) *matched = r.second;
        return 0;
    });
}
uint64_t tvara_kv_book_prefix_reuse(tvara_kv_book* b, const int32_t* tokens, size_t token_count, int partial,
                                    size_t* reused) {
    return guarded<uint64_t>(0, [&] {
        if (!tokens && token_count) throw std::invalid_argument("invalid token buffer");
        const auto r = b->prefixes().reuse({tokens, token_count}, partial != 0);
        if (reused) *reused = r.second;
        return r.first;
    });
}
int tvara_kv_book_prefix_pin(tvara_kv_book* b, uint64_t node) {
    return guarded<int>(-1, [&] {
        b->prefixes().pin(node);
        return 0;
    });
}
int tvara_kv_book_prefix_unpin(tvara_kv_book* b, uint64_t node) {
    return guarded<int>(-1, [&] {
        b->prefixes().unpin(node);
        return 0;
    });
}
int tvara_kv_book_prefix_touch(tvara_kv_book* b, uint64_t node) {
    return guarded<int>(-1, [&] {
        b->prefixes().touch(node);
        return 0;
    });
}
int tvara_kv_book_prefix_evict_one(tvara_kv_book* b) {
    return guarded<int>(-1, [&] { return b->prefixes().evict_one() ? 1 : 0; });
}
size_t tvara_kv_book_prefix_size(tvara_kv_book* b) {
    return guarded<size_t>(0, [&] { return b->prefixes().size(); });
}

}  // extern "C"
