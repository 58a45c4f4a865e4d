// shim_program.cpp -- a host program written against include/iam_b200.hpp the way the
// reference's own drivers are written against bucket_mul.hpp / model.hpp / the layer classes
// (test_generation.cpp, per-layer drivers).  Built and run by tests/test_shim_program_gpu.py,
// which writes the inputs and checks every output against the CPU oracle.
//
//   shim_program <dir>
//
// <dir>/bm_in.bin     int32 in_dim, int32 out_dim, f32 effort, f32 x[in], u16 stats[16 in],
//                     u16 probes[in], u16 buckets[16 in][out / 16]
// <dir>/model_in.bin  int32 dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab,
//                     max_ctx, tied; f32 norm_eps; f64 rope_theta; u64 seed; f32 effort;
//                     int32 n_tok; int32 tokens[n_tok]; int32 block_pos; f32 x[dim]; f32 h[dim]
// Outputs (raw little-endian arrays):
//   bm_full.bin, bm_two_step.bin          BucketMul::fullMul and calcDispatch + mul, f32[out]
//   model_logits.bin, model_sel.bin       MistralModel::forward per token: f32[n_tok][vocab], i64[n_tok]
//   layer_out.bin, layer_counts.bin, layer_k.bin, layer_v.bin
//                                         TransformerLayer(0)::forward(x) at block_pos: f32[dim],
//                                         i32[7] selected rows per matrix, layer 0's K/V cache
//   attn_out.bin, attn_counts.bin, attn_k.bin, attn_v.bin
//                                         Attention(1)::forward(h) at block_pos, layer 1's cache
//   ffn_out.bin, ffn_counts.bin           FeedForward(1)::forward(h)
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <vector>

#include "iam_b200.hpp"

using namespace iam_shim;

namespace {

struct Reader {
    std::vector<char> data;
    size_t at = 0;
    explicit Reader(const std::string& path) {
        std::ifstream f(path, std::ios::binary);
        if (!f) throw std::runtime_error("cannot open " + path);
        data.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
    }
    template <typename T>
    T get() {
        T v;
        take(&v, sizeof(T));
        return v;
    }
    template <typename T>
    std::vector<T> vec(size_t n) {
        std::vector<T> v(n);
        take(v.data(), n * sizeof(T));
        return v;
    }
    void take(void* dst, size_t n) {
        if (at + n > data.size()) throw std::runtime_error("input file too short");
        std::memcpy(dst, data.data() + at, n);
        at += n;
    }
};

template <typename T>
void write(const std::string& path, const std::vector<T>& v) {
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(v.data()), (std::streamsize)(v.size() * sizeof(T)));
    if (!f) throw std::runtime_error("cannot write " + path);
}

std::vector<int> counts_of(MistralModel& m, int layer) {
    std::vector<int> all((size_t)m.cfg.n_layers * 7);
    check(iam_model_selected_rows_by_matrix(m.handle, all.data(), (int)all.size()), "selected_rows_by_matrix");
    return std::vector<int>(all.begin() + 7 * layer, all.begin() + 7 * layer + 7);
}

std::vector<uint16_t> cache_of(MistralModel& m, int layer, int which) {
    size_t bytes = 0;
    check(iam_model_read_weight(m.handle, layer, which, nullptr, 0, &bytes), "read_weight size");
    std::vector<uint16_t> v(bytes / 2);
    check(iam_model_read_weight(m.handle, layer, which, v.data(), bytes, nullptr), "read_weight");
    return v;
}

void run_bucketmul(Gpu& gpu, const std::string& dir) {
    Reader r(dir + "/bm_in.bin");
    const int in = r.get<int32_t>(), out = r.get<int32_t>();
    const float effort = r.get<float>();
    const int cols = out / 16;
    BufferWrapper<float> x(&gpu, (size_t)in), y(&gpu, (size_t)out);
    BufferWrapper<uint16_t> stats(&gpu, std::vector<size_t>{(size_t)16 * in, 1});
    BufferWrapper<uint16_t> probes(&gpu, (size_t)in);
    BufferWrapper<uint16_t> buckets(&gpu, std::vector<size_t>{(size_t)16 * in, (size_t)cols});
    x.setData(&gpu, r.vec<float>(in));
    stats.setData(&gpu, r.vec<uint16_t>((size_t)16 * in));
    probes.setData(&gpu, r.vec<uint16_t>(in));
    buckets.setData(&gpu, r.vec<uint16_t>((size_t)16 * in * cols));

    BucketMul* bm = BucketMul::shared(&gpu);
    y.zero(&gpu);  // callers zero the output first, as attention.hpp:157-159 does
    bm->fullMul(&x, &stats, &probes, &buckets, 0, in, cols, in, effort, &y);
    write(dir + "/bm_full.bin", y.getData(&gpu));
    y.zero(&gpu);
    bm->calcDispatch(&x, &stats, &probes, 0, in, cols, in, effort);
    bm->mul(&buckets, &y);
    write(dir + "/bm_two_step.bin", y.getData(&gpu));
}

void run_model(Gpu& gpu, const std::string& dir) {
    Reader r(dir + "/model_in.bin");
    iam_model_config c{};
    c.dim = r.get<int32_t>();
    c.n_layers = r.get<int32_t>();
    c.n_heads = r.get<int32_t>();
    c.n_kv_heads = r.get<int32_t>();
    c.head_dim = r.get<int32_t>();
    c.ffn_dim = r.get<int32_t>();
    c.vocab = r.get<int32_t>();
    c.max_ctx = r.get<int32_t>();
    c.tied_embeddings = r.get<int32_t>();
    c.norm_eps = r.get<float>();
    c.rope_theta = r.get<double>();
    const unsigned long long seed = r.get<uint64_t>();
    const float effort = r.get<float>();
    const int n_tok = r.get<int32_t>();
    const std::vector<int32_t> tokens = r.vec<int32_t>(n_tok);
    const int block_pos = r.get<int32_t>();
    const std::vector<float> xin = r.vec<float>(c.dim), hin = r.vec<float>(c.dim);

    MistralModel model(&gpu, c, seed);
    BufferWrapper<float> logits(&gpu, (size_t)c.vocab);
    std::vector<float> all_logits;
    std::vector<long long> sel;
    model.reset_caches();
    for (int i = 0; i < n_tok; ++i) {  // test_generation.cpp:202-213: one forward per token
        model.forward(tokens[i], i, effort, &logits);
        const std::vector<float> l = logits.getData(&gpu);
        all_logits.insert(all_logits.end(), l.begin(), l.end());
        long long s = 0;
        check(iam_model_selected_rows(model.handle, &s), "selected_rows");
        sel.push_back(s);
    }
    write(dir + "/model_logits.bin", all_logits);
    write(dir + "/model_sel.bin", sel);

    BufferWrapper<float> x(&gpu, (size_t)c.dim), h(&gpu, (size_t)c.dim), y(&gpu, (size_t)c.dim);
    x.setData(&gpu, xin);
    h.setData(&gpu, hin);

    TransformerLayer layer0(&gpu, &model, 0);
    layer0.forward(&x, 0, block_pos, effort, &y);
    write(dir + "/layer_out.bin", y.getData(&gpu));
    write(dir + "/layer_counts.bin", counts_of(model, 0));
    write(dir + "/layer_k.bin", cache_of(model, 0, IAM_W_K_CACHE));
    write(dir + "/layer_v.bin", cache_of(model, 0, IAM_W_V_CACHE));

    Attention attn1(&gpu, &model, 1);
    y.zero(&gpu);
    attn1.forward(&h, 1, block_pos, effort, &y);
    write(dir + "/attn_out.bin", y.getData(&gpu));
    write(dir + "/attn_counts.bin", counts_of(model, 1));
    write(dir + "/attn_k.bin", cache_of(model, 1, IAM_W_K_CACHE));
    write(dir + "/attn_v.bin", cache_of(model, 1, IAM_W_V_CACHE));

    FeedForward ffn1(&gpu, &model, 1);
    y.zero(&gpu);
    ffn1.forward(&h, &y, effort);
    write(dir + "/ffn_out.bin", y.getData(&gpu));
    write(dir + "/ffn_counts.bin", counts_of(model, 1));
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: %s <dir>\n", argv[0]);
        return 2;
    }
    try {
        Gpu gpu(0);
        run_bucketmul(gpu, argv[1]);
        run_model(gpu, argv[1]);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "shim_program: %s\n", e.what());
        return 1;
    }
    return 0;
}
