// Engine: loading, KV pool, and the ragged step.
#include "engine.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <set>

#include "attention_plan.hpp"
#include <cstdlib>

#include "collective.hpp"
#include "p2p_allreduce.hpp"
#include "tp_plan.hpp"

namespace tvara {
namespace {

std::size_t align256(std::size_t n) { return (n + 255) & ~std::size_t(255); }

struct Segment {
    std::string name;
    int row0, rows, col0, cols;
};

// Raw GGUF rows of one or more tensors (same type and width), optionally
// interleaving two tensors row by row (gate/up).
struct RawMatrix {
    int type = 0, rows = 0, cols = 0;
    std::vector<std::uint8_t> bytes;
};

RawMatrix gather(const gguf::File& f, const std::vector<Segment>& segs, bool interleave) {
    RawMatrix m;
    m.type = static_cast<int>(f.info(segs[0].name).type);
    m.cols = segs[0].cols;
    std::size_t elems = 0, width = 0;
    if (!block_shape(m.type, elems, width)) throw std::invalid_argument("unsupported native weight type");
    if (m.cols % elems) throw std::invalid_argument("tensor-parallel split is not a whole number of blocks");
    const std::size_t out_row = std::size_t(m.cols) / elems * width;
    for (const auto& s : segs) {
        if (static_cast<int>(f.info(s.name).type) != m.type || s.cols != m.cols)
            throw std::invalid_argument("fused tensors must share type and width");
        m.rows += s.rows;
    }
    m.bytes.resize(std::size_t(m.rows) * out_row);
    std::size_t r_out = 0;
    std::vector<std::span<const std::byte>> payloads;
    for (const auto& s : segs) payloads.push_back(f.payload(s.name));
    auto copy_row = [&](std::size_t si, int r, std::size_t dst_row) {
        const auto& s = segs[si];
        const auto& info = f.info(s.name);
        const std::size_t in_row = std::size_t(info.dims[0]) / elems * width;
        const std::size_t off = std::size_t(s.row0 + r) * in_row + std::size_t(s.col0) / elems * width;
        std::memcpy(m.bytes.data() + dst_row * out_row, payloads[si].data() + off, out_row);
    };
    if (interleave) {
        for (int r = 0; r < segs[0].rows; ++r)
            for (std::size_t si = 0; si < segs.size(); ++si) copy_row(si, r, r_out++);
    } else {
        for (std::size_t si = 0; si < segs.size(); ++si)
            for (int r = 0; r < segs[si].rows; ++r) copy_row(si, r, r_out++);
    }
    return m;
}

std::size_t matrix_bytes(int type, int rows, int cols) {
    return align256(qs_row_bytes(type, cols) * rows) + align256(meta_row_bytes(type, cols) * rows) + align256(rows);
}

}  // namespace

Engine::Engine(const std::string& path, std::size_t max_blocks, std::size_t block_tokens, const EngineOptions& opt)
    : opt_(opt) {
    if (opt.device >= 0) TVARA_CUDA(cudaSetDevice(opt.device));
    TVARA_CUDA(cudaGetDevice(&device_));
    gguf::File f(path);
    cfg_ = gguf::llama_config(f.doc());
    gguf::validate_llama_tensors(f.doc(), cfg_);
    metadata_ = f.metadata_json();
    const int tp = std::max(1, opt.tp_size);
    const TpShard shard = tp_shard(f, cfg_, opt.tp_rank, tp);
    hidden_ = int(cfg_.hidden);
    vocab_ = int(cfg_.vocab);
    layers_ = int(cfg_.layers);
    dim_ = shard.head_dim;
    hq_ = shard.heads;
    hkv_ = shard.kv_heads;
    ffn_ = shard.ffn;
    qkv_w_ = (hq_ + 2 * hkv_) * dim_;
    // the LM head splits by vocabulary rows under tensor parallelism
    head_ld_ = (vocab_ + tp - 1) / tp;
    head_row0_ = opt.tp_rank * head_ld_;
    head_rows_ = std::min(head_ld_, vocab_ - head_row0_);
    if (head_rows_ < 1) throw std::invalid_argument("tensor-parallel size exceeds the vocabulary");
    if (dim_ != 16 && dim_ != 32 && dim_ != 64 && dim_ != 128 && dim_ != 256)
        throw std::invalid_argument("unsupported head_dim (16, 32, 64, 128, 256)");
    tmax_ = std::max(1, opt.max_step_tokens);

    CacheGeometry g{cfg_.layers, cfg_.kv_heads, cfg_.head_dim(), block_tokens, max_blocks};
    book_ = std::make_unique<SequenceBook>(g);
    radix_ = std::make_unique<PrefixTrie>(*book_, "tvara-b200-engine");

    TVARA_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    if (tp > 1) {
        if (!opt.has_nccl_id) throw std::invalid_argument("tensor parallelism needs an NCCL unique id");
        coll_ = std::make_unique<Collective>(opt.nccl_id.data(), opt.tp_rank, tp);
    }
    try {
        load(f);
    } catch (...) {
        if (weights_) cudaFree(weights_);
        if (planes_) cudaFree(planes_);
        weights_ = nullptr;
        planes_ = nullptr;
        cudaStreamDestroy(stream_);
        throw;
    }
}

Engine::~Engine() {
    if (stream_) cudaStreamSynchronize(stream_);
    for (auto e : events_) cudaEventDestroy(e);
    radix_.reset();
    peer_.reset();  // closes the peers' buffers before this rank's scratch is freed
    coll_.reset();
    for (void* p : {static_cast<void*>(weights_), static_cast<void*>(planes_), static_cast<void*>(rope_cos_), static_cast<void*>(rope_sin_), kv_, static_cast<void*>(token_ids_), static_cast<void*>(kv_scales_),
                    static_cast<void*>(x_), static_cast<void*>(meta_dev_), static_cast<void*>(err_), tc_ws_, sample_buf_})
        if (p) cudaFree(p);
    if (meta_host_) cudaFreeHost(meta_host_);
    if (err_host_) cudaFreeHost(err_host_);
    if (stream_) cudaStreamDestroy(stream_);
}

void Engine::load(const gguf::File& f) {
    const int r = opt_.tp_rank, tp = std::max(1, opt_.tp_size);
    const int D = hidden_, d = dim_;
    const bool tied = !f.has("output.weight");
    // ---- plan every device matrix
    struct Plan {
        std::vector<Segment> segs;
        bool interleave = false;
        DeviceMatrix* out = nullptr;
    };
    std::vector<Plan> plans;
    std::vector<std::pair<std::string, const float**>> norms;
    lw_.assign(layers_, {});
    plans.push_back({{{"token_embd.weight", 0, vocab_, 0, D}}, false, &embed_});
    if (!tied || tp > 1)  // this rank's vocabulary rows of the head (all of them at tp 1)
        plans.push_back({{{tied ? "token_embd.weight" : "output.weight", head_row0_, head_rows_, 0, D}}, false, &head_});
    norms.push_back({"output_norm.weight", &final_norm_});
    auto type_of = [&](const std::string& n) { return static_cast<int>(f.info(n).type); };
    for (int l = 0; l < layers_; ++l) {
        const auto p = "blk." + std::to_string(l) + ".";
        auto& L = lw_[l];
        norms.push_back({p + "attn_norm.weight", &L.attn_norm});
        norms.push_back({p + "ffn_norm.weight", &L.ffn_norm});
        const Segment sq{p + "attn_q.weight", r * hq_ * d, hq_ * d, 0, D};
        const Segment sk{p + "attn_k.weight", r * hkv_ * d, hkv_ * d, 0, D};
        const Segment sv{p + "attn_v.weight", r * hkv_ * d, hkv_ * d, 0, D};
        if (type_of(sq.name) == type_of(sk.name) && type_of(sq.name) == type_of(sv.name)) {
            L.qkv.resize(1);
            plans.push_back({{sq, sk, sv}, false, &L.qkv[0]});
        } else {
            L.qkv.resize(3);
            plans.push_back({{sq}, false, &L.qkv[0]});
            plans.push_back({{sk}, false, &L.qkv[1]});
            plans.push_back({{sv}, false, &L.qkv[2]});
        }
        plans.push_back({{{p + "attn_output.weight", 0, D, r * hq_ * d, hq_ * d}}, false, &L.o});
        const Segment sg{p + "ffn_gate.weight", r * ffn_, ffn_, 0, D};
        const Segment su{p + "ffn_up.weight", r * ffn_, ffn_, 0, D};
        if (type_of(sg.name) == type_of(su.name)) {
            L.gateup.resize(1);
            plans.push_back({{sg, su}, true, &L.gateup[0]});
        } else {
            gate_up_fused_ = false;
            L.gateup.resize(2);
            plans.push_back({{sg}, false, &L.gateup[0]});
            plans.push_back({{su}, false, &L.gateup[1]});
        }
        plans.push_back({{{p + "ffn_down.weight", 0, D, r * ffn_, ffn_}}, false, &L.down});
    }
    // ---- sizes: one allocation for every matrix, norm and the rope tables
    std::size_t total = 0, staging = 0;
    for (const auto& pl : plans) {
        int rows = 0;
        for (const auto& s : pl.segs) rows += s.rows;
        const int type = type_of(pl.segs[0].name);
        total += matrix_bytes(type, rows, pl.segs[0].cols);
        std::size_t e = 0, w = 0;
        block_shape(type, e, w);
        staging = std::max(staging, std::size_t(rows) * (pl.segs[0].cols / e) * w);
    }
    for (const auto& n : norms) {
        total += align256(std::size_t(D) * 4);
        staging = std::max(staging, gguf::tensor_bytes(f.info(n.first)));
    }
    weight_bytes_ = total;
    TVARA_CUDA(cudaMalloc(&weights_, total));
    std::uint8_t* staging_dev = nullptr;
    TVARA_CUDA(cudaMalloc(&staging_dev, align256(staging)));
    std::uint8_t* cursor = weights_;
    int* flag = nullptr;
    TVARA_CUDA(cudaMalloc(&flag, sizeof(int)));
    TVARA_CUDA(cudaMemset(flag, 0, sizeof(int)));
    try {
        for (const auto& pl : plans) {
            RawMatrix raw = gather(f, pl.segs, pl.interleave);
            TVARA_CUDA(cudaMemcpyAsync(staging_dev, raw.bytes.data(), raw.bytes.size(), cudaMemcpyHostToDevice, stream_));
            DeviceMatrix m;
            m.type = raw.type;
            m.rows = raw.rows;
            m.cols = raw.cols;
            m.qs_row = qs_row_bytes(raw.type, raw.cols);
            m.meta_row = meta_row_bytes(raw.type, raw.cols);
            std::uint8_t* qs = cursor;
            cursor += align256(m.qs_row * m.rows);
            std::uint8_t* meta = cursor;
            cursor += align256(m.meta_row * m.rows);
            launch_repack(raw.type, staging_dev, raw.rows, raw.cols, qs, meta, stream_);
            m.qs = qs;
            m.meta = meta;
            auto* shifts = reinterpret_cast<signed char*>(cursor);
            cursor += align256(m.rows);
            launch_row_shift(m, shifts, stream_);
            m.row_shift = shifts;
            launch_finite_check(m, flag, stream_);
            *pl.out = m;
            TVARA_CUDA(cudaStreamSynchronize(stream_));  // raw host buffer is released next iteration
        }
        for (const auto& n : norms) {
            const auto& info = f.info(n.first);
            auto bytes = f.payload(n.first);
            TVARA_CUDA(cudaMemcpyAsync(staging_dev, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, stream_));
            std::size_t e = 0, w = 0;
            if (!block_shape(static_cast<int>(info.type), e, w)) throw std::invalid_argument("unsupported native weight type");
            float* out = reinterpret_cast<float*>(cursor);
            cursor += align256(std::size_t(D) * 4);
            launch_dequantize(static_cast<int>(info.type), staging_dev, std::size_t(D) / e, out, stream_);
            DeviceMatrix nm;
            nm.type = kF32;
            nm.rows = 1;
            nm.cols = D;
            nm.qs = reinterpret_cast<const std::uint8_t*>(out);
            nm.qs_row = std::size_t(D) * 4;
            launch_finite_check(nm, flag, stream_);
            *n.second = out;
        }
        if (tied && tp == 1) head_ = embed_;
        int bad = 0;
        TVARA_CUDA(cudaMemcpyAsync(&bad, flag, sizeof(int), cudaMemcpyDeviceToHost, stream_));
        TVARA_CUDA(cudaStreamSynchronize(stream_));
        if (bad) throw std::invalid_argument("nonfinite model weight");
    } catch (...) {
        cudaFree(staging_dev);
        cudaFree(flag);
        throw;
    }
    cudaFree(staging_dev);
    cudaFree(flag);

    // ---- tensor-core forms of the projections: Q4_K rows as sc*q built
    // from the packed rows inside the kernel, with block scales and the min
    // term in side arrays (about 0.16 bytes per weight beside the packed
    // 0.5625; two MMAs per K-step), other types as exact FP16 hi/lo planes of
    // their values (4 bytes per weight, the footprint of the reference's own
    // F32 expansion); batches of <= 4 tokens keep streaming the packed rows.
    if (opt_.weight_planes != 2) {
        std::vector<DeviceMatrix*> mats;
        for (auto& L : lw_) {
            for (auto& m : L.qkv) mats.push_back(&m);
            mats.push_back(&L.o);
            for (auto& m : L.gateup) mats.push_back(&m);
            mats.push_back(&L.down);
        }
        mats.push_back(&head_);
        // Q4_K rows: the two-MMA factorisation, from the packed rows (side
        // arrays only; default) or from a prebuilt FP16 plane of sc*q (mode 4)
        auto q4k_form = [&](const DeviceMatrix* m) {
            return opt_.weight_planes != 3 && m->type == kQ4_K && m->cols % 256 == 0;
        };
        const bool q4k_plane = opt_.weight_planes == 4;
        auto form_bytes = [&](const DeviceMatrix* m) -> std::size_t {
            if (q4k_form(m))
                return ((q4k_plane ? q4k_planes_bytes(m->rows, m->cols) : q4k_packed_form_bytes(m->rows, m->cols)) +
                        255) & ~std::size_t(255);
            return m->cols % 32 == 0 ? std::size_t(m->rows) * m->cols * 4 : 0;
        };
        std::size_t need = 0;
        for (auto* m : mats) need += form_bytes(m);
        const std::size_t es = opt_.kv_elem_bytes();
        const std::size_t pool = std::size_t(layers_) * 2 * hkv_ * book_->geometry().tokens_per_block * d * es *
                                 book_->geometry().max_blocks;
        std::size_t free_b = 0, total_b = 0;
        TVARA_CUDA(cudaMemGetInfo(&free_b, &total_b));
        const std::size_t reserve = std::size_t(4) << 30;  // scratch, workspaces, other users
        const bool fits = need + pool + reserve <= free_b;
        if (opt_.weight_planes == 1 && !fits) throw std::runtime_error("weight planes do not fit in device memory");
        if (fits && need) {
            TVARA_CUDA(cudaMalloc(&planes_, need));
            plane_bytes_ = need;
            auto* at = reinterpret_cast<unsigned char*>(planes_);
            for (auto* m : mats) {
                const std::size_t bytes = form_bytes(m);
                if (!bytes) continue;
                if (q4k_form(m)) {
                    if (q4k_plane) launch_q4k_planes(*m, at, stream_);
                    else launch_q4k_packed_form(*m, at, stream_);
                } else {
                    const std::size_t n = std::size_t(m->rows) * m->cols;
                    auto* p = reinterpret_cast<std::uint16_t*>(at);
                    launch_planes(*m, p, p + n, stream_);
                    m->plane_hi = p;
                    m->plane_lo = p + n;
                }
                at += bytes;
            }
            TVARA_CUDA(cudaStreamSynchronize(stream_));
        }
    }

    // ---- RoPE table with the reference's float expression (model.hpp:71-72)
    const std::size_t half = d / 2;
    std::vector<float> cs(cfg_.context * half), sn(cfg_.context * half);
    for (std::size_t p = 0; p < cfg_.context; ++p)
        for (std::size_t i = 0; i < half; ++i) {
            const float angle = static_cast<float>(p) / std::pow(cfg_.theta, static_cast<float>(2 * i) / static_cast<float>(d));
            cs[p * half + i] = std::cos(angle);
            sn[p * half + i] = std::sin(angle);
        }
    TVARA_CUDA(cudaMalloc(&rope_cos_, cs.size() * 4));
    TVARA_CUDA(cudaMalloc(&rope_sin_, sn.size() * 4));
    TVARA_CUDA(cudaMemcpy(rope_cos_, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    TVARA_CUDA(cudaMemcpy(rope_sin_, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));

    // ---- KV pool: [block][layer][K|V][kv head][slot][d]
    const auto& g = book_->geometry();
    const std::size_t es = opt_.kv_elem_bytes();
    kind_stride_ = (long long)hkv_ * g.tokens_per_block * d;
    layer_stride_ = 2 * kind_stride_;
    block_stride_ = (long long)layers_ * layer_stride_;
    const std::size_t pool_bytes = std::size_t(block_stride_) * es * g.max_blocks;
    std::size_t free_b = 0, total_b = 0;
    TVARA_CUDA(cudaMemGetInfo(&free_b, &total_b));
    if (pool_bytes > free_b) throw std::runtime_error("KV pool does not fit in device memory");
    TVARA_CUDA(cudaMalloc(&kv_, pool_bytes));
    TVARA_CUDA(cudaMalloc(&token_ids_, g.max_blocks * g.tokens_per_block * sizeof(int)));
    if (opt_.kv_i8) TVARA_CUDA(cudaMalloc(&kv_scales_, std::size_t(block_stride_ / d) * g.max_blocks * sizeof(float)));

    // ---- scratch for tmax_ tokens (one allocation)
    const std::size_t T = tmax_;
    partial_cap_ = 8192;
    const std::size_t ff_w = std::size_t(ffn_) * (gate_up_fused_ ? 1 : 2);
    const std::size_t split_head = tp > 1 ? T * std::size_t(head_ld_) * tp + T * vocab_ +
                                                T * argmax_part_bytes() * (tp + 1) / 4 + 64 * 3
                                          : 0;
    const std::size_t floats = T * D * 2 + T * qkv_w_ + T * hq_ * d * 2 + T * ff_w + T * vocab_ +
                               partial_cap_ * hq_ * (d + 2) + 64 * 8 + split_head;
    std::size_t bytes = floats * 4 + T * 4 + 4096;
    TVARA_CUDA(cudaMalloc(&x_, bytes));
    float* c = x_;
    auto take = [&](std::size_t n) {
        float* p = c;
        c += (n + 63) & ~std::size_t(63);
        return p;
    };
    x_ = take(T * D);
    xn_ = take(T * D);
    qkv_ = take(T * qkv_w_);
    q_ = take(T * hq_ * d);
    att_ = take(T * hq_ * d);
    ff_ = take(T * ffn_);
    ffu_ = gate_up_fused_ ? nullptr : take(T * ffn_);
    logits_ = take(T * vocab_);
    partial_ = take(partial_cap_ * hq_ * (d + 2));
    argmax_ = reinterpret_cast<unsigned*>(take(T));
    if (tp > 1) {
        gather_ = take(T * std::size_t(head_ld_) * tp);
        full_ = take(T * vocab_);
        amparts_ = take(T * argmax_part_bytes() * (tp + 1) / 4);
    }
    const int max_k = std::max({D, hq_ * d, ffn_});
    tc_ws_bytes_ = gemm_tc_workspace(int(T), max_k);
    TVARA_CUDA(cudaMalloc(&tc_ws_, tc_ws_bytes_));
    TVARA_CUDA(cudaMalloc(&err_, sizeof(int)));
    TVARA_CUDA(cudaMemset(err_, 0, sizeof(int)));
    TVARA_CUDA(cudaHostAlloc(&err_host_, sizeof(int), cudaHostAllocDefault));
    // tensor parallelism: the residual x_ (the start of the scratch, at the
    // same offset on every rank) is summed over NVLink peer memory; callers
    // may keep NCCL's allreduce with TVARA_ALLREDUCE=nccl (every rank must
    // see the same setting)
    if (coll_) {
        const char* mode = std::getenv("TVARA_ALLREDUCE");
        if (!(mode && std::string(mode) == "nccl"))
            peer_ = std::make_unique<PeerAllreduce>(*coll_, x_, T * std::size_t(D), stream_);
    }
}

void Engine::allreduce_residual(std::size_t n) {
    if (peer_ && peer_->applies(x_, n)) peer_->allreduce_sum(x_, n, err_, stream_);
    else coll_->allreduce_sum(x_, n, stream_);
}

void Engine::projection(const DeviceMatrix& w, const float* x, int ldx, int tokens, float* y, int ldy, int epi,
                        bool presplit) {
    GemmArgs a;
    a.w = w;
    a.presplit = presplit;
    a.x = x;
    a.ldx = ldx;
    a.tokens = tokens;
    a.y = y;
    a.ldy = ldy;
    a.epilogue = epi;
    a.err = err_;
    launch_projection(a, tc_ws_, tc_ws_bytes_, stream_);
}

void Engine::step(std::span<const std::uint64_t> seqs, std::span<const std::uint32_t> cu,
                  std::span<const std::uint32_t> tokens, bool all_logits, float* logits, std::uint32_t* argmax,
                  bool finite_argmax, const SampleSpec* sample) {
    finite_argmax_ = finite_argmax;
    sample_ = sample;
    const std::size_t n = seqs.size();
    if (sample && all_logits) throw std::invalid_argument("device sampling takes one row per sequence");
    if (sample && (sample->top_k < 0 || sample->top_k > kSampleMaxK || std::size_t(sample->top_k) > cfg_.vocab))
        throw std::invalid_argument("top-k candidates must be between 0 and 64");
    if (!n || cu.size() != n + 1 || cu[0] != 0) throw std::invalid_argument("invalid batch layout");
    for (std::size_t i = 0; i < n; ++i)
        if (cu[i + 1] <= cu[i]) throw std::invalid_argument("invalid batch layout");
    if (tokens.size() != cu[n]) throw std::invalid_argument("invalid batch layout");
    {
        std::set<std::uint64_t> uniq(seqs.begin(), seqs.end());
        if (uniq.size() != n) throw std::invalid_argument("sequence listed twice in one step");
    }
    std::vector<std::size_t> entry(n);
    for (std::size_t i = 0; i < n; ++i) {
        entry[i] = book_->sequence(seqs[i]).length;
        const std::size_t count = cu[i + 1] - cu[i];
        if (entry[i] + count > cfg_.context) throw std::invalid_argument("paged decode exceeds token/context limits");
        if (sample && entry[i] + count > kSampleHistoryMax)
            throw std::invalid_argument("device sampling holds at most 16384 tokens of history");
        for (std::size_t j = cu[i]; j < cu[i + 1]; ++j)
            if (tokens[j] >= cfg_.vocab) throw std::invalid_argument("paged decode exceeds token/context limits");
    }
    // ---- accounting: all-or-nothing over the call
    const std::size_t T = tokens.size();
    const std::size_t tpb = book_->geometry().tokens_per_block;
    std::vector<int> blk(T), slot(T);
    std::vector<int2> copies;
    std::size_t touched = 0;
    try {
        for (std::size_t i = 0; i < n; ++i) {
            touched = i + 1;
            for (std::size_t j = cu[i]; j < cu[i + 1]; ++j) {
                BlockCopy c{SIZE_MAX, SIZE_MAX};
                book_->append(seqs[i], &c);
                if (c.from != SIZE_MAX) copies.push_back(make_int2(int(c.from), int(c.to)));
                const auto& t = book_->sequence(seqs[i]);
                blk[j] = int(t.blocks.back().id);
                slot[j] = int((t.length - 1) % tpb);
            }
        }
    } catch (...) {
        if (!copies.empty()) {  // replacement blocks stay in the tables: give them their data
            int2* dev = nullptr;
            if (cudaMalloc(&dev, copies.size() * sizeof(int2)) == cudaSuccess) {
                cudaMemcpy(dev, copies.data(), copies.size() * sizeof(int2), cudaMemcpyHostToDevice);
                copy_blocks(dev, int(copies.size()));
                cudaStreamSynchronize(stream_);
                cudaFree(dev);
            }
        }
        for (std::size_t i = 0; i < touched; ++i) book_->truncate(seqs[i], entry[i]);
        throw;
    }
    acc_h2d_ = acc_d2h_ = 0;
    try {
        // ---- split into device sub-steps of at most tmax_ tokens
        std::size_t i = 0, j = 0;  // sequence, token offset within it
        bool first = true;
        const std::size_t rows_total = all_logits ? T : n;
        while (i < n) {
            Sub sub;
            if (first) sub.copies = copies;
            first = false;
            std::size_t room = std::size_t(tmax_);
            std::vector<std::size_t> seq_ids;
            while (i < n && room) {
                const std::size_t count = cu[i + 1] - cu[i];
                const std::size_t take = std::min(room, count - j);
                const int si = int(seq_ids.size());
                seq_ids.push_back(i);
                const auto& table = book_->sequence(seqs[i]);
                sub.table_off.push_back(int(sub.tables.size()));
                for (auto b : table.blocks) sub.tables.push_back(int(b.id));
                for (std::size_t k = 0; k < take; ++k) {
                    const std::size_t g = cu[i] + j + k;
                    sub.tok.push_back(int(tokens[g]));
                    sub.pos.push_back(int(entry[i] + j + k));
                    sub.blk.push_back(blk[g]);
                    sub.slot.push_back(slot[g]);
                    sub.seq_of.push_back(si);
                    const bool last = j + k + 1 == count;
                    if (all_logits || last) {
                        sub.out_rows.push_back(int(sub.tok.size() - 1));
                        sub.out_dest.push_back(all_logits ? (long long)g : (long long)i);
                    }
                }
                room -= take;
                j += take;
                if (j == count) {
                    ++i;
                    j = 0;
                }
            }
            run(sub, logits, argmax, rows_total);
        }
        last_h2d_ = acc_h2d_;
        last_d2h_ = acc_d2h_;
    } catch (...) {
        cudaStreamSynchronize(stream_);
        for (std::size_t k = 0; k < n; ++k) book_->truncate(seqs[k], entry[k]);
        throw;
    }
}

template <class F>
void Engine::timed(int cls, F&& launch) {
    if (!profiling_) {
        launch();
        return;
    }
    if (2 * event_used_ + 2 > events_.size()) {
        for (int i = 0; i < 64; ++i) {
            cudaEvent_t e;
            TVARA_CUDA(cudaEventCreate(&e));
            events_.push_back(e);
        }
        event_class_.resize(events_.size() / 2);
    }
    TVARA_CUDA(cudaEventRecord(events_[2 * event_used_], stream_));
    launch();
    TVARA_CUDA(cudaEventRecord(events_[2 * event_used_ + 1], stream_));
    event_class_[event_used_++] = cls;
}

void Engine::profile_collect() {
    for (std::size_t i = 0; i < event_used_; ++i) {
        float ms = 0.f;
        TVARA_CUDA(cudaEventElapsedTime(&ms, events_[2 * i], events_[2 * i + 1]));
        prof_ms_[event_class_[i]] += ms;
        ++prof_n_[event_class_[i]];
    }
    event_used_ = 0;
}

void Engine::set_profiling(bool on) {
    profiling_ = on;
    host_idle_valid_ = false;
    for (int i = 0; i < kProfClasses; ++i) {
        prof_ms_[i] = 0;
        prof_n_[i] = 0;
    }
}

void Engine::profile_read(double* ms, unsigned long long* groups) const {
    for (int i = 0; i < kProfClasses; ++i) {
        if (ms) ms[i] = prof_ms_[i];
        if (groups) groups[i] = prof_n_[i];
    }
}

void Engine::copy_blocks(const int2* pairs, int n) {
    launch_block_copy(kv_, block_stride_ * (long long)opt_.kv_elem_bytes(), pairs, n, stream_);
    if (kv_scales_) launch_id_copy(reinterpret_cast<int*>(kv_scales_), int(block_stride_ / cfg_.head_dim()), pairs, n, stream_);
    launch_id_copy(token_ids_, int(book_->geometry().tokens_per_block), pairs, n, stream_);
}

void Engine::reserve(std::uint64_t seq, std::size_t count) {
    const std::size_t entry = book_->sequence(seq).length;
    if (count > cfg_.context - entry) throw std::invalid_argument("paged decode exceeds token/context limits");
    std::vector<int2> copies;
    auto copy_now = [&] {
        if (copies.empty()) return;
        int2* dev = nullptr;
        TVARA_CUDA(cudaMalloc(&dev, copies.size() * sizeof(int2)));
        TVARA_CUDA(cudaMemcpy(dev, copies.data(), copies.size() * sizeof(int2), cudaMemcpyHostToDevice));
        copy_blocks(dev, int(copies.size()));
        TVARA_CUDA(cudaStreamSynchronize(stream_));
        cudaFree(dev);
    };
    try {
        for (std::size_t i = 0; i < count; ++i) {
            BlockCopy c{SIZE_MAX, SIZE_MAX};
            book_->append(seq, &c);
            if (c.from != SIZE_MAX) copies.push_back(make_int2(int(c.from), int(c.to)));
        }
    } catch (...) {
        copy_now();
        book_->truncate(seq, entry);
        throw;
    }
    copy_now();
    // reserved positions hold no token: id -1 (the sampler's history skips them)
    const auto& t = book_->sequence(seq);
    const std::size_t tpb = book_->geometry().tokens_per_block;
    for (std::size_t p = entry; p < entry + count;) {
        const std::size_t b = p / tpb, end = std::min(entry + count, (b + 1) * tpb);
        TVARA_CUDA(cudaMemsetAsync(token_ids_ + t.blocks[b].id * tpb + p % tpb, 0xFF, (end - p) * sizeof(int), stream_));
        p = end;
    }
    TVARA_CUDA(cudaStreamSynchronize(stream_));
}

void Engine::run(Sub& s, float* logits, std::uint32_t* argmax, std::size_t) {
    const int T = int(s.tok.size());
    const int d = dim_, D = hidden_;
    const int tpb = int(book_->geometry().tokens_per_block);
    // ---- attention work list
    std::vector<int> vis(T), toff(T);
    for (int t = 0; t < T; ++t) {
        vis[t] = s.pos[t] + 1;
        toff[t] = s.table_off[s.seq_of[t]];
    }
    AttnPlan plan = plan_attention(vis, toff, tpb, hkv_, partial_cap_, 148,
                                   attention_chunk_rows(opt_.kv_i8 ? 2 : opt_.kv_f16 ? 1 : 0, d, hq_ / hkv_, tpb));
    auto& work = plan.work;
    auto& comb = plan.comb;
    auto& wpart = plan.part;
    // ---- pack metadata into one pinned buffer and upload
    const int R = int(s.out_rows.size());
    // device sampler inputs per output row k (sequence s.out_dest[k])
    const SampleSpec* sp = sample_;
    const int words = int((vocab_ + 31) / 32);
    std::vector<int> smp_hlen, smp_toff;
    std::vector<double> smp_par;
    int hist_cap = 1;
    if (sp && R > 0) {
        smp_hlen.resize(R);
        smp_toff.resize(R);
        smp_par.resize(std::size_t(R) * 3);
        for (int k = 0; k < R; ++k) {
            const int o = s.out_rows[k];
            const auto i = s.out_dest[k];
            smp_hlen[k] = s.pos[o] + 1;
            smp_toff[k] = s.table_off[s.seq_of[o]];
            smp_par[3 * k] = sp->repetition ? sp->repetition[i] : 1.0;
            smp_par[3 * k + 1] = sp->frequency ? sp->frequency[i] : 0.0;
            smp_par[3 * k + 2] = sp->presence ? sp->presence[i] : 0.0;
            while (hist_cap < smp_hlen[k]) hist_cap <<= 1;
        }
        const int K = sp->top_k;
        const std::size_t bytes = std::size_t(R) * (4 + std::size_t(K) * 12) + std::size_t(R) * hist_cap * 8 + 256;
        if (bytes > sample_cap_) {
            TVARA_CUDA(cudaStreamSynchronize(stream_));
            if (sample_buf_) cudaFree(sample_buf_);
            sample_buf_ = nullptr;
            sample_cap_ = 0;
            TVARA_CUDA(cudaMalloc(&sample_buf_, bytes * 2));
            sample_cap_ = bytes * 2;
        }
    }
    const std::size_t need = std::size_t(T) * 4 + s.tables.size() + work.size() * 5 + comb.size() * 4 +
                             plan.chunk.size() * 4 + 4 +
                             s.copies.size() * 2 + R + 64 +
                             (sp ? std::size_t(R) * (8 + (sp->allowed ? words : 0)) + 16 : 0);
    if (need > meta_cap_) {
        TVARA_CUDA(cudaStreamSynchronize(stream_));
        if (meta_dev_) cudaFree(meta_dev_);
        if (meta_host_) cudaFreeHost(meta_host_);
        meta_cap_ = std::max(need * 2, std::size_t(1) << 16);
        TVARA_CUDA(cudaMalloc(&meta_dev_, meta_cap_ * 4));
        TVARA_CUDA(cudaHostAlloc(&meta_host_, meta_cap_ * 4, cudaHostAllocDefault));
    } else {
        TVARA_CUDA(cudaStreamSynchronize(stream_));  // previous step done with the host mirror
    }
    std::size_t at = 0;
    auto put = [&](const void* src, std::size_t ints) -> int* {
        at = (at + 3) & ~std::size_t(3);  // 16-byte alignment for int4 arrays
        std::memcpy(meta_host_ + at, src, ints * 4);
        int* dev = meta_dev_ + at;
        at += ints;
        return dev;
    };
    int* d_tok = put(s.tok.data(), T);
    int* d_pos = put(s.pos.data(), T);
    int* d_blk = put(s.blk.data(), T);
    int* d_slot = put(s.slot.data(), T);
    int* d_tables = put(s.tables.data(), s.tables.size());
    int4* d_work = reinterpret_cast<int4*>(put(work.data(), work.size() * 4));
    int* d_wpart = put(wpart.data(), wpart.size());
    int4* d_comb = reinterpret_cast<int4*>(put(comb.data(), comb.size() * 4));
    int4* d_chunk = reinterpret_cast<int4*>(put(plan.chunk.data(), plan.chunk.size() * 4));
    int2* d_copy = reinterpret_cast<int2*>(put(s.copies.data(), s.copies.size() * 2));
    int* d_rows = put(s.out_rows.data(), R);
    int *d_hlen = nullptr, *d_toff = nullptr;
    const double* d_par = nullptr;
    const unsigned* d_allow = nullptr;
    if (sp && R > 0) {
        d_hlen = put(smp_hlen.data(), R);
        d_toff = put(smp_toff.data(), R);
        d_par = reinterpret_cast<const double*>(put(smp_par.data(), std::size_t(R) * 6));
        if (sp->allowed) {
            at = (at + 3) & ~std::size_t(3);
            for (int k = 0; k < R; ++k)
                std::memcpy(meta_host_ + at + std::size_t(k) * words, sp->allowed + std::size_t(s.out_dest[k]) * words,
                            std::size_t(words) * 4);
            d_allow = reinterpret_cast<const unsigned*>(meta_dev_ + at);
            at += std::size_t(R) * words;
        }
    }
    if (profiling_ && host_idle_valid_) {
        prof_ms_[kProfHost] +=
            std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - host_idle_since_).count();
        ++prof_n_[kProfHost];
    }
    TVARA_CUDA(cudaMemcpyAsync(meta_dev_, meta_host_, at * 4, cudaMemcpyHostToDevice, stream_));
    acc_h2d_ += at * 4;

    event_used_ = 0;
    timed(kProfOther, [&] {
        copy_blocks(d_copy, int(s.copies.size()));
        launch_embed(embed_, d_tok, T, x_, D, stream_, token_ids_, d_blk, d_slot,
                     int(book_->geometry().tokens_per_block));
    });
    // RMSNorm whose every consumer takes the tensor-core path also writes
    // their split input (one kernel instead of a norm and a split per
    // projection); the F32 output is written in every case.
    auto norm = [&](const float* w, const int* rows, int n, const std::vector<const DeviceMatrix*>& consumers) {
        bool tc = tc_ws_ != nullptr;
        for (const auto* m : consumers) tc = tc && gemm_tc_supported(*m, n);
        if (tc) launch_rmsnorm_split(x_, D, rows, n, D, w, cfg_.eps, xn_, D, tc_ws_, tc_ws_bytes_, stream_);
        else launch_rmsnorm(x_, D, rows, n, D, w, cfg_.eps, xn_, D, stream_);
        return tc;
    };
    for (int l = 0; l < layers_; ++l) {
        const auto& L = lw_[l];
        std::vector<const DeviceMatrix*> qkv_in, gu_in;
        for (const auto& m : L.qkv) qkv_in.push_back(&m);
        for (const auto& m : L.gateup) gu_in.push_back(&m);
        bool split = false;
        timed(kProfOther, [&] { split = norm(L.attn_norm, nullptr, T, qkv_in); });
        timed(kProfProjection, [&] {
            if (L.qkv.size() == 1) {
                projection(L.qkv[0], xn_, D, T, qkv_, qkv_w_, kStore, split);
            } else {
                projection(L.qkv[0], xn_, D, T, qkv_, qkv_w_, kStore, split);
                projection(L.qkv[1], xn_, D, T, qkv_ + hq_ * d, qkv_w_, kStore, split);
                projection(L.qkv[2], xn_, D, T, qkv_ + (hq_ + hkv_) * d, qkv_w_, kStore, split);
            }
        });
        RopeArgs ra;
        ra.qkv = qkv_;
        ra.ldqkv = qkv_w_;
        ra.q = q_;
        ra.tokens = T;
        ra.hq = hq_;
        ra.hkv = hkv_;
        ra.dim = d;
        ra.interleaved = cfg_.interleaved;
        ra.cosines = rope_cos_;
        ra.sines = rope_sin_;
        ra.positions = d_pos;
        ra.slot_block = d_blk;
        ra.slot_index = d_slot;
        ra.kv = kv_;
        ra.kv_f16 = opt_.kv_f16;
        ra.kv_i8 = opt_.kv_i8;
        ra.kv_scales = kv_scales_;
        ra.block_stride = block_stride_;
        ra.layer_offset = (long long)l * layer_stride_;
        ra.kind_stride = kind_stride_;
        ra.tpb = tpb;
        ra.max_blocks = int(book_->geometry().max_blocks);
        ra.err = err_;
        timed(kProfOther, [&] { launch_rope_kv(ra, stream_); });
        AttnArgs aa;
        aa.q = q_;
        aa.out = att_;
        aa.kv = kv_;
        aa.kv_f16 = opt_.kv_f16;
        aa.kv_i8 = opt_.kv_i8;
        aa.kv_scales = kv_scales_;
        aa.hq = hq_;
        aa.hkv = hkv_;
        aa.dim = d;
        aa.tpb = tpb;
        aa.block_stride = block_stride_;
        aa.layer_offset = (long long)l * layer_stride_;
        aa.kind_stride = kind_stride_;
        aa.tables = d_tables;
        aa.work = d_work;
        aa.work_part = d_wpart;
        aa.n_work = int(work.size());
        aa.partial = partial_;
        aa.combine = d_comb;
        aa.n_combine = int(comb.size());
        aa.chunk_work = d_chunk;
        aa.n_chunk = int(plan.chunk.size());
        aa.max_blocks = int(book_->geometry().max_blocks);
        aa.err = err_;
        timed(kProfAttention, [&] { launch_attention(aa, stream_); });
        const bool lead = opt_.tp_rank == 0;
        // Under tensor parallelism rank 0 adds its partial to the residual and
        // the others store theirs, so the sum over ranks is x + sum(partials).
        timed(kProfProjection, [&] { projection(L.o, att_, hq_ * d, T, x_, D, lead ? kAdd : kStore); });
        if (coll_) timed(kProfCollective, [&] { allreduce_residual(std::size_t(T) * D); });
        timed(kProfOther, [&] { split = norm(L.ffn_norm, nullptr, T, gu_in); });
        timed(kProfProjection, [&] {
            if (L.gateup.size() == 1) {
                projection(L.gateup[0], xn_, D, T, ff_, ffn_, kSwiGLU, split);
            } else {
                projection(L.gateup[0], xn_, D, T, ff_, ffn_, kStore, split);
                projection(L.gateup[1], xn_, D, T, ffu_, ffn_, kStore, split);
                launch_swiglu(ff_, ffu_, T * ffn_, stream_);
            }
        });
        timed(kProfProjection, [&] { projection(L.down, ff_, ffn_, T, x_, D, lead ? kAdd : kStore); });
        if (coll_) timed(kProfCollective, [&] { allreduce_residual(std::size_t(T) * D); });
    }
    if (R > 0) {
        timed(kProfHead, [&] {
            const bool hsplit = norm(final_norm_, d_rows, R, {&head_});
            const float* rows_full = logits_;  // [R][vocab] where the sampler reads
            if (!coll_) {
                projection(head_, xn_, D, R, logits_, vocab_, kStore, hsplit);
                if (argmax) launch_argmax(logits_, R, vocab_, argmax_, finite_argmax_, stream_);
            } else {
                // this rank's vocabulary slice; only argmax records (and, when
                // asked for, the logits) cross NVLink
                const int tp = coll_->size();
                projection(head_, xn_, D, R, logits_, head_ld_, kStore, hsplit);
                if (argmax) {
                    auto* mine = static_cast<unsigned char*>(amparts_);
                    auto* all = mine + std::size_t(R) * argmax_part_bytes();
                    launch_argmax_part(logits_, R, head_ld_, head_rows_, head_row0_, mine, stream_);
                    coll_->allgather(mine, all, std::size_t(R) * argmax_part_bytes(), stream_);
                    launch_argmax_merge(all, R, tp, argmax_, finite_argmax_, stream_);
                }
                if (logits || sp) coll_->allgather(logits_, gather_, std::size_t(R) * head_ld_ * 4, stream_);
                if (sp) {
                    for (int k = 0; k < tp; ++k) {
                        const int cols = std::min(head_ld_, vocab_ - k * head_ld_);
                        TVARA_CUDA(cudaMemcpy2DAsync(full_ + std::size_t(k) * head_ld_, std::size_t(vocab_) * 4,
                                                     gather_ + std::size_t(k) * R * head_ld_, std::size_t(head_ld_) * 4,
                                                     std::size_t(cols) * 4, R, cudaMemcpyDeviceToDevice, stream_));
                    }
                    rows_full = full_;
                }
            }
            if (sp) {
                SampleJob job;
                job.logits = rows_full;
                job.ld = vocab_;
                job.rows = R;
                job.vocab = vocab_;
                job.ids = token_ids_;
                job.tables = d_tables;
                job.toff = d_toff;
                job.tpb = int(book_->geometry().tokens_per_block);
                job.hlen = d_hlen;
                job.hist_cap = hist_cap;
                job.params = d_par;
                job.allowed = d_allow;
                job.words = words;
                job.top_k = sp->top_k;
                auto* b = static_cast<unsigned char*>(sample_buf_);
                job.pen = reinterpret_cast<double*>(b);
                job.pen_stride = hist_cap;
                b += std::size_t(R) * hist_cap * 8;
                job.top_val = reinterpret_cast<double*>(b);
                b += std::size_t(R) * sp->top_k * 8;
                job.status = reinterpret_cast<int*>(b);
                b += std::size_t(R) * 4;
                job.top_id = reinterpret_cast<unsigned*>(b);
                job.argmax = argmax_;
                launch_sample(job, stream_);
            }
        });
    }
    TVARA_CUDA(cudaMemcpyAsync(err_host_, err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    // ---- results to the caller: contiguous destination runs, one copy each
    acc_d2h_ += sizeof(int);
    std::vector<unsigned> am(argmax || sp ? R : 0);
    if ((argmax || sp) && R) {
        TVARA_CUDA(cudaMemcpyAsync(am.data(), argmax_, R * 4, cudaMemcpyDeviceToHost, stream_));
        acc_d2h_ += std::uint64_t(R) * 4;
    }
    const int K = sp ? sp->top_k : 0;
    std::vector<int> st(sp ? R : 0);
    std::vector<double> tv(std::size_t(R) * K);
    std::vector<unsigned> ti(std::size_t(R) * K);
    if (sp && R) {
        const auto* b = static_cast<const unsigned char*>(sample_buf_) + std::size_t(R) * hist_cap * 8;
        if (K) {
            TVARA_CUDA(cudaMemcpyAsync(tv.data(), b, tv.size() * 8, cudaMemcpyDeviceToHost, stream_));
            TVARA_CUDA(cudaMemcpyAsync(ti.data(), b + std::size_t(R) * K * 8 + std::size_t(R) * 4, ti.size() * 4,
                                       cudaMemcpyDeviceToHost, stream_));
        }
        TVARA_CUDA(cudaMemcpyAsync(st.data(), b + std::size_t(R) * K * 8, std::size_t(R) * 4, cudaMemcpyDeviceToHost,
                                   stream_));
        acc_d2h_ += std::uint64_t(R) * (4 + std::uint64_t(K) * 12);
    }
    if (logits) acc_d2h_ += std::uint64_t(R) * vocab_ * 4;
    if (logits) {
        int k = 0;
        while (k < R) {
            int e = k + 1;
            while (e < R && s.out_dest[e] == s.out_dest[e - 1] + 1) ++e;
            if (!coll_) {
                TVARA_CUDA(cudaMemcpyAsync(logits + s.out_dest[k] * vocab_, logits_ + (long long)k * vocab_,
                                           std::size_t(e - k) * vocab_ * 4, cudaMemcpyDeviceToHost, stream_));
            } else {
                for (int r = 0; r < coll_->size(); ++r) {  // rank r's columns of rows k..e
                    const int cols = std::min(head_ld_, vocab_ - r * head_ld_);
                    TVARA_CUDA(cudaMemcpy2DAsync(logits + s.out_dest[k] * vocab_ + std::size_t(r) * head_ld_,
                                                 std::size_t(vocab_) * 4,
                                                 gather_ + (std::size_t(r) * R + k) * head_ld_, std::size_t(head_ld_) * 4,
                                                 std::size_t(cols) * 4, e - k, cudaMemcpyDeviceToHost, stream_));
                }
            }
            k = e;
        }
    }
    TVARA_CUDA(cudaStreamSynchronize(stream_));
    profile_collect();  // before the idle stamp: reading the events is profiling cost, not the step's
    host_idle_since_ = std::chrono::steady_clock::now();
    host_idle_valid_ = true;
    if (*err_host_) {
        const int code = *err_host_;
        TVARA_CUDA(cudaMemsetAsync(err_, 0, sizeof(int), stream_));
        if (code == 3) throw std::invalid_argument("Nonfinite KV input");
        if (code == 5) throw std::runtime_error("tensor-parallel peer did not reach the allreduce (wait timed out)");
        throw std::runtime_error("device bounds check failed (code " + std::to_string(code) + ")");
    }
    if (argmax)
        for (int k = 0; k < R; ++k) argmax[s.out_dest[k]] = am[k];
    if (sp)
        for (int k = 0; k < R; ++k) {
            const auto i = s.out_dest[k];
            if (sp->argmax) sp->argmax[i] = am[k];
            if (sp->status) sp->status[i] = st[k];
            for (int c = 0; c < K; ++c) {
                if (sp->top_values) sp->top_values[i * K + c] = tv[std::size_t(k) * K + c];
                if (sp->top_ids) sp->top_ids[i * K + c] = ti[std::size_t(k) * K + c];
            }
        }
}

}  // namespace tvara
