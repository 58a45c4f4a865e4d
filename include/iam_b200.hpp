// iam_b200.hpp -- header-only C++ shim over libiamb200.so that keeps the reference's host
// API: the class and method names of bucket_mul.hpp (BufferWrapper, ScalarFloat, BucketMul),
// model.hpp (MistralModel) and the layer classes (TransformerLayer, Attention, FeedForward of
// transformer_layer.hpp, attention.hpp, feedforward.hpp), so the reference's callers
// (test_generation.cpp, per-layer drivers) compile against it with their OpenCL Gpu* replaced
// by a device id.
//
// Differences from the reference, all deliberate:
//   - buffers are CUDA device allocations (cudaMalloc) instead of cl_mem;
//   - BucketMul is one handle per shim instance (shared() keeps the singleton convention);
//   - errors throw std::runtime_error carrying iam_last_error() (the reference swallows
//     clSetKernelArg errors, bucket_mul.hpp:167-173);
//   - every call is asynchronous on the shim's stream; eval() synchronises (gpu.hpp:399-447).
#ifndef IAM_B200_HPP
#define IAM_B200_HPP

#include <cuda_runtime.h>

#include <cassert>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "iam_b200.h"

namespace iam_shim {

inline void check(int rc, const char* what) {
    if (rc != IAM_OK) throw std::runtime_error(std::string(what) + ": " + iam_last_error());
}

inline void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Stand-in for the reference's Gpu object (gpu.hpp:81-589): a device and a stream.
struct Gpu {
    int device = 0;
    cudaStream_t stream = nullptr;
    explicit Gpu(int dev = 0) : device(dev) {
        check_cuda(cudaSetDevice(dev), "cudaSetDevice");
        check_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
    }
    ~Gpu() {
        if (stream) cudaStreamDestroy(stream);
    }
    void eval() { check_cuda(cudaStreamSynchronize(stream), "eval"); }
};

// bucket_mul.hpp:13-67
template <typename T>
class BufferWrapper {
   public:
    size_t count, rows, cols, byte_size;
    T* buffer = nullptr;
    Gpu* gpu_ref;

    BufferWrapper(Gpu* gpu, size_t size) : count(size), rows(size), cols(1), byte_size(size * sizeof(T)), gpu_ref(gpu) {
        check_cuda(cudaMalloc(&buffer, byte_size ? byte_size : sizeof(T)), "BufferWrapper cudaMalloc");
    }
    BufferWrapper(Gpu* gpu, const std::vector<size_t>& shape)
        : count(calculateSize(shape)),
          rows(shape.size() > 0 ? shape[0] : 1),
          cols(shape.size() > 1 ? shape[1] : 1),
          byte_size(calculateSize(shape) * sizeof(T)),
          gpu_ref(gpu) {
        check_cuda(cudaMalloc(&buffer, byte_size ? byte_size : sizeof(T)), "BufferWrapper cudaMalloc");
    }
    BufferWrapper(const BufferWrapper&) = delete;
    BufferWrapper& operator=(const BufferWrapper&) = delete;
    ~BufferWrapper() { cudaFree(buffer); }

    void zero(Gpu* gpu) { check_cuda(cudaMemsetAsync(buffer, 0, byte_size, gpu->stream), "zero"); }
    std::vector<T> getData(Gpu* gpu) {
        gpu->eval();
        std::vector<T> data(count);
        check_cuda(cudaMemcpy(data.data(), buffer, byte_size, cudaMemcpyDeviceToHost), "getData");
        return data;
    }
    T get(Gpu* gpu, size_t index) { return getData(gpu)[index]; }
    void setData(Gpu* gpu, const std::vector<T>& data) {
        assert(data.size() == count);  // bucket_mul.hpp:55
        check_cuda(cudaMemcpyAsync(buffer, data.data(), byte_size, cudaMemcpyHostToDevice, gpu->stream), "setData");
        gpu->eval();
    }
    static size_t calculateSize(const std::vector<size_t>& shape) {
        size_t s = 1;
        for (size_t d : shape) s *= d;
        return s;
    }
};

// bucket_mul.hpp:69-84
class ScalarFloat : public BufferWrapper<float> {
   public:
    explicit ScalarFloat(Gpu* gpu, float value = 0.0f) : BufferWrapper<float>(gpu, 1) { setData(gpu, {value}); }
    float getValue(Gpu* gpu) { return get(gpu, 0); }
};

// bucket_mul.hpp:99-268.  stats may be the file layout [R][4] (the reference's) or a packed
// channel-3 array [R]; the layout is inferred from the buffer's cols (4 or 1).
class BucketMul {
   public:
    static constexpr int PROBES_COUNT = IAM_PROBES_COUNT;
    Gpu* gpu;
    iam_bucketmul_t handle = nullptr;

    static BucketMul* shared(Gpu* g) {
        static BucketMul instance(g);
        return &instance;
    }
    explicit BucketMul(Gpu* g) : gpu(g) { check(iam_bucketmul_create(&handle, g->device), "BucketMul"); }
    ~BucketMul() { iam_bucketmul_destroy(handle); }

    void calcDispatch(BufferWrapper<float>* input, BufferWrapper<uint16_t>* stats, BufferWrapper<uint16_t>* probes,
                      int expertNo, int inSize, int bucketCols, int expertSize, float effort) {
        check(iam_bucketmul_calc_dispatch(handle, input->buffer, stats->buffer, stats->cols == 1 ? 1 : 4,
                                          probes->buffer, expertNo, inSize, bucketCols, expertSize, effort, gpu->stream),
              "BucketMul::calcDispatch");
    }
    void mul(BufferWrapper<uint16_t>* buckets, BufferWrapper<float>* output) {
        check(iam_bucketmul_mul(handle, buckets->buffer, (int)buckets->rows, (int)buckets->cols, output->buffer,
                                gpu->stream),
              "BucketMul::mul");
    }
    void fullMul(BufferWrapper<float>* input, BufferWrapper<uint16_t>* stats, BufferWrapper<uint16_t>* probes,
                 BufferWrapper<uint16_t>* buckets, int expertNo, int inSize, int bucketCols, int expertSize,
                 float effort, BufferWrapper<float>* output) {
        check(iam_bucketmul_full(handle, input->buffer, stats->buffer, stats->cols == 1 ? 1 : 4, probes->buffer,
                                 buckets->buffer, expertNo, inSize, bucketCols, expertSize, effort, output->buffer,
                                 nullptr, nullptr, gpu->stream),
              "BucketMul::fullMul");
    }
};

// model.hpp:15-238 with the dimensions as a config (the reference hard-codes Mistral-7B).
class MistralModel {
   public:
    Gpu* gpu;
    iam_model_t handle = nullptr;
    iam_model_config cfg;

    static iam_model_config mistral7b(int vocab = 32768, int max_ctx = 2048) {
        iam_model_config c{};
        c.dim = 4096;
        c.n_layers = 32;
        c.n_heads = 32;
        c.n_kv_heads = 8;
        c.head_dim = 128;
        c.ffn_dim = 14336;
        c.vocab = vocab;
        c.max_ctx = max_ctx;
        c.norm_eps = 1e-5f;
        c.rope_theta = 1e6;
        c.tied_embeddings = 0;
        return c;
    }
    MistralModel(Gpu* g, const std::string& weights_dir, const iam_model_config& c = mistral7b()) : gpu(g), cfg(c) {
        check(iam_model_load(&handle, weights_dir.c_str(), &cfg, g->device), "MistralModel");
    }
    // A model of random N(0, 0.02) weights (no counterpart in the reference: tests, benchmarks).
    MistralModel(Gpu* g, const iam_model_config& c, unsigned long long seed) : gpu(g), cfg(c) {
        check(iam_model_create_random(&handle, &cfg, seed, g->device), "MistralModel (random)");
    }
    MistralModel(const MistralModel&) = delete;
    MistralModel& operator=(const MistralModel&) = delete;
    ~MistralModel() { iam_model_destroy(handle); }
    // model.hpp:152-231 (no eval inside; call gpu->eval() or read the logits)
    void forward(int token_id, int pos, float effort, BufferWrapper<float>* logits_out) {
        check(iam_model_forward(handle, token_id, pos, effort, logits_out ? logits_out->buffer : nullptr, gpu->stream),
              "MistralModel::forward");
    }
    void reset_caches() {
        check(iam_model_reset(handle, gpu->stream), "MistralModel::reset_caches");
        gpu->eval();
    }
    // The whole prompt in one batched pass on the dense tensor-core path, in place of one
    // forward() per prompt token (test_generation.cpp:202-213); returns the greedy next token.
    int prefill(const int* tokens, int n_tokens, int start_pos, BufferWrapper<float>* logits_out) {
        int next = -1;
        check(iam_model_prefill(handle, tokens, n_tokens, start_pos, logits_out ? logits_out->buffer : nullptr,
                                &next, gpu->stream),
              "MistralModel::prefill");
        return next;
    }
};

// transformer_layer.hpp:15-122: a decoder layer of a MistralModel (its weights, gains and KV
// cache).  The reference's caller-owned caches and temporaries are accepted and not used: the
// layer reads and writes the model's own KV cache of layer_idx.
class TransformerLayer {
   public:
    Gpu* gpu;
    MistralModel* model;
    int layer;
    TransformerLayer(Gpu* g, MistralModel* m, int layer_idx) : gpu(g), model(m), layer(layer_idx) {}
    void forward(BufferWrapper<float>* input, int layer_idx, int pos, float effort, BufferWrapper<float>* output) {
        check(iam_layer_forward(model->handle, layer_idx, input->buffer, pos, effort, output->buffer, gpu->stream),
              "TransformerLayer::forward");
    }
    // the reference's argument list (transformer_layer.hpp:75-93)
    void forward(BufferWrapper<float>* input, int layer_idx, int pos, float effort, BufferWrapper<float>* /*k_cache*/,
                 BufferWrapper<float>* /*v_cache*/, BufferWrapper<float>* /*h_norm*/,
                 BufferWrapper<float>* /*temp_xq*/, BufferWrapper<float>* /*temp_xk*/,
                 BufferWrapper<float>* /*temp_xv*/, BufferWrapper<float>* /*temp_xk_repeated*/,
                 BufferWrapper<float>* /*temp_xq_heads*/, BufferWrapper<float>* /*temp_xk_heads*/,
                 BufferWrapper<float>* /*temp_scores*/, BufferWrapper<float>* /*temp_attn_output*/,
                 BufferWrapper<float>* /*attn_out*/, BufferWrapper<float>* /*fxn*/, BufferWrapper<float>* /*ffn_out*/,
                 BufferWrapper<float>* output) {
        forward(input, layer_idx, pos, effort, output);
    }
};

// attention.hpp:19-202: q/k/v bucketMuls, RoPE, the fp16 K/V append at pos, attention over
// [0, pos] and the o bucketMul of an already normalised input; no residual.
class Attention {
   public:
    Gpu* gpu;
    MistralModel* model;
    int layer;
    Attention(Gpu* g, MistralModel* m, int layer_idx) : gpu(g), model(m), layer(layer_idx) {}
    void forward(BufferWrapper<float>* input, int layer_idx, int pos, float effort, BufferWrapper<float>* output) {
        check(iam_attention_forward(model->handle, layer_idx, input->buffer, pos, effort, output->buffer, gpu->stream),
              "Attention::forward");
    }
    // the reference's argument list (attention.hpp:135-149)
    void forward(BufferWrapper<float>* input, int layer_idx, int pos, float effort, BufferWrapper<float>* /*k_cache*/,
                 BufferWrapper<float>* /*v_cache*/, BufferWrapper<float>* /*temp_xq*/,
                 BufferWrapper<float>* /*temp_xk*/, BufferWrapper<float>* /*temp_xv*/,
                 BufferWrapper<float>* /*temp_xk_repeated*/, BufferWrapper<float>* /*temp_xq_heads*/,
                 BufferWrapper<float>* /*temp_xk_heads*/, BufferWrapper<float>* /*temp_scores*/,
                 BufferWrapper<float>* /*temp_attn_output*/, BufferWrapper<float>* output) {
        forward(input, layer_idx, pos, effort, output);
    }
};

// feedforward.hpp:14-183: down(SiLU(gate(x)) * up(x)) of an already normalised input.
class FeedForward {
   public:
    Gpu* gpu;
    MistralModel* model;
    int layer;
    FeedForward(Gpu* g, MistralModel* m, int layer_idx) : gpu(g), model(m), layer(layer_idx) {}
    void forward(BufferWrapper<float>* input, BufferWrapper<float>* output, float effort = 1.0f) {
        check(iam_feedforward_forward(model->handle, layer, input->buffer, effort, output->buffer, gpu->stream),
              "FeedForward::forward");
    }
};

}  // namespace iam_shim

#endif  // IAM_B200_HPP
