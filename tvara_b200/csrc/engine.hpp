// The B200 decode/prefill engine behind the C ABI: packed weights and the
// paged KV pool in HBM, host-side block accounting, and one device step per
// ragged batch (the reference's PagedModelExecutor::decode, paged_model.hpp:
// 12-28, for many sequences and tokens at once).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <array>
#include <chrono>
#include <memory>
#include <span>
#include <string>
#include <vector>

#include "common.hpp"
#include "gguf.hpp"
#include "kernels.cuh"
#include "kvbook.hpp"
#include "p2p_allreduce.hpp"

namespace tvara {

struct EngineOptions {
    int device = -1;
    bool kv_f16 = false;
    bool kv_i8 = false;  // int8 per token-head with F32 scales (quantized_kv.py)
    std::size_t kv_elem_bytes() const { return kv_i8 ? 1 : kv_f16 ? 2 : 4; }
    int max_step_tokens = 2048;
    int tp_rank = 0, tp_size = 1;
    bool has_nccl_id = false;
    std::array<char, 128> nccl_id{};
    // Exact FP16 hi/lo planes of the projections for the tensor-core path:
    // 0 = when they fit beside the KV pool, 1 = always, 2 = never, 3 = the
    // hi/lo planes for every type (no Q4_K form), when they fit.
    int weight_planes = 0;
};

class Collective;  // NCCL communicator of a tensor-parallel group (collective.cpp)

// Device-side logit post-processing of a step's rows (k_sample.cu); all
// arrays are host memory indexed by the step's sequence order.
struct SampleSpec {
    const double* repetition = nullptr;   // null: 1
    const double* frequency = nullptr;    // null: 0
    const double* presence = nullptr;     // null: 0
    const std::uint32_t* allowed = nullptr;  // [n][ceil(vocab / 32)] or null
    int top_k = 0;
    std::uint32_t* argmax = nullptr;      // [n]
    std::int32_t* status = nullptr;       // [n]
    double* top_values = nullptr;         // [n][top_k]
    std::uint32_t* top_ids = nullptr;     // [n][top_k]
};
constexpr std::size_t kSampleHistoryMax = 16384;  // tokens of history the device sampler holds per row

struct LayerWeights {
    const float* attn_norm = nullptr;
    const float* ffn_norm = nullptr;
    std::vector<DeviceMatrix> qkv;     // one fused matrix, or q, k, v
    DeviceMatrix o;
    std::vector<DeviceMatrix> gateup;  // interleaved gate/up rows, or gate, up
    DeviceMatrix down;
};

class Engine {
public:
    Engine(const std::string& path, std::size_t max_blocks, std::size_t block_tokens, const EngineOptions& opt);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    const gguf::LlamaConfig& config() const { return cfg_; }
    const std::string& metadata() const { return metadata_; }
    SequenceBook& book() { return *book_; }
    PrefixTrie& radix() { return *radix_; }
    const EngineOptions& options() const { return opt_; }

    // One ragged step; see tvara_batch_step.  Rows of logits / argmax are
    // written to host memory (either may be null).  finite_argmax marks rows
    // whose logits are not all finite with argmax 0xFFFFFFFF.
    void step(std::span<const std::uint64_t> seqs, std::span<const std::uint32_t> cu,
              std::span<const std::uint32_t> tokens, bool all_logits, float* logits, std::uint32_t* argmax,
              bool finite_argmax = false, const SampleSpec* sample = nullptr);

    // Appends positions to a sequence's table without computing K/V.
    void reserve(std::uint64_t seq, std::size_t count);
    void* kv_pool() const { return kv_; }
    float* kv_scales() const { return kv_scales_; }
    long long block_elements() const { return block_stride_; }
    int local_kv_heads() const { return hkv_; }

    // Device bytes of the packed weights and of the FP16 planes (0 if none).
    std::size_t weight_bytes() const { return weight_bytes_; }
    std::size_t plane_bytes() const { return plane_bytes_; }

    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

    // Device time per kernel class, measured with CUDA events on the engine
    // stream around each launch group while enabled (off by default).
    // kProfHost: host time with the stream idle, from the end of one device
    // step (its results back on the host) to the first work of the next one.
    enum ProfileClass {
        kProfAttention = 0,
        kProfProjection,
        kProfHead,
        kProfOther,
        kProfCollective,
        kProfHost,
        kProfClasses
    };
    void set_profiling(bool on);
    void profile_read(double* ms, unsigned long long* groups) const;
    std::uint64_t last_h2d() const { return last_h2d_; }
    std::uint64_t last_d2h() const { return last_d2h_; }

private:
    template <class F>
    void timed(int cls, F&& launch);
    void profile_collect();
    bool profiling_ = false;
    bool host_idle_valid_ = false;
    std::chrono::steady_clock::time_point host_idle_since_;
    std::uint64_t last_h2d_ = 0, last_d2h_ = 0, acc_h2d_ = 0, acc_d2h_ = 0;
    std::vector<cudaEvent_t> events_;
    std::vector<int> event_class_;
    std::size_t event_used_ = 0;
    double prof_ms_[kProfClasses] = {};
    unsigned long long prof_n_[kProfClasses] = {};

    struct Sub {  // one device launch sequence over <= max_step_tokens tokens
        std::vector<int> tok, pos, blk, slot;
        std::vector<int> seq_of;           // index into the sub-step's sequence list
        std::vector<int> table_off;        // per sequence
        std::vector<int> tables;
        std::vector<int> out_rows;         // token indices whose logits are wanted
        std::vector<long long> out_dest;   // destination row in the caller's buffer
        std::vector<int2> copies;
    };
    void load(const gguf::File& f);
    DeviceMatrix upload_matrix(const gguf::File& f, const std::string& name, int row0, int rows, int col0, int cols,
                               std::uint8_t*& cursor);
    void run(Sub& sub, float* logits, std::uint32_t* argmax, std::size_t vocab_rows_total);
    // presplit: the tensor-core input is already in the workspace (launch_rmsnorm_split)
    void projection(const DeviceMatrix& w, const float* x, int ldx, int tokens, float* y, int ldy, int epi,
                    bool presplit = false);

    gguf::LlamaConfig cfg_;
    EngineOptions opt_;
    std::string metadata_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    std::unique_ptr<SequenceBook> book_;
    std::unique_ptr<PrefixTrie> radix_;
    std::unique_ptr<Collective> coll_;
    std::unique_ptr<PeerAllreduce> peer_;  // tensor-parallel residual sums over peer memory
    void allreduce_residual(std::size_t n);

    // local (per tensor-parallel rank) shapes
    int hq_ = 0, hkv_ = 0, dim_ = 0, ffn_ = 0, hidden_ = 0, vocab_ = 0, layers_ = 0, qkv_w_ = 0;
    // LM head rows of this rank: [head_row0_, head_row0_ + head_rows_) of the
    // vocabulary (all of it without tensor parallelism); head_ld_ = the
    // per-rank slice width every rank's logits buffer is laid out with
    int head_row0_ = 0, head_rows_ = 0, head_ld_ = 0;
    bool gate_up_fused_ = true;

    // device memory
    std::uint8_t* weights_ = nullptr;
    std::size_t weight_bytes_ = 0;
    std::uint16_t* planes_ = nullptr;  // FP16 hi/lo planes of the projections (optional)
    std::size_t plane_bytes_ = 0;
    DeviceMatrix embed_, head_;
    const float* final_norm_ = nullptr;
    std::vector<LayerWeights> lw_;
    float* rope_cos_ = nullptr;
    float* rope_sin_ = nullptr;
    void* kv_ = nullptr;
    long long block_stride_ = 0, layer_stride_ = 0, kind_stride_ = 0;
    // Token id of every KV slot, [block][slot]: the history the device-side
    // sampler reads through a sequence's block table.
    int* token_ids_ = nullptr;
    float* kv_scales_ = nullptr;  // int8 pools: one F32 scale per (block, layer, kind, head, slot) row
    // Copies blocks (KV payload and token ids) on the engine stream.
    void copy_blocks(const int2* pairs, int n);

    int tmax_ = 0;
    float *x_ = nullptr, *xn_ = nullptr, *qkv_ = nullptr, *q_ = nullptr, *att_ = nullptr, *ff_ = nullptr,
          *ffu_ = nullptr, *logits_ = nullptr, *partial_ = nullptr, *xo_ = nullptr;
    // tensor parallelism: every rank's logits slices ([rank][row][head_ld_]),
    // the rows reassembled ([row][vocab], for the sampler), argmax records
    float *gather_ = nullptr, *full_ = nullptr;
    void* amparts_ = nullptr;
    unsigned* argmax_ = nullptr;
    bool finite_argmax_ = false;
    const SampleSpec* sample_ = nullptr;  // during a sampling step
    void* sample_buf_ = nullptr;          // status, top-k and penalty scratch of the sampler
    std::size_t sample_cap_ = 0;
    int* err_ = nullptr;
    void* tc_ws_ = nullptr;        // tensor-core projection: hi/lo FP16 activations + token scales
    std::size_t tc_ws_bytes_ = 0;
    std::size_t partial_cap_ = 0;  // partial rows (part x hq)
    // per-step metadata (device + pinned host mirror)
    int* meta_dev_ = nullptr;
    int* meta_host_ = nullptr;
    std::size_t meta_cap_ = 0;     // ints
    int* err_host_ = nullptr;
};

}  // namespace tvara
