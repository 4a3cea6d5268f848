// The C++ face on the device: a Qwen-3.5-shaped state owner runs one attention
// layer (prefill, then a decode step) and one delta-rule layer (chunked
// prefill, clear, again), and a Gemma-shaped cache runs a sliding-window layer
// whose batch is longer than its window.  Inputs come from fp32 files in the
// directory given as argv[1]; outputs go back there for the Python side to
// compare with the oracle.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <string>
#include <vector>

#include "nmg.hpp"

namespace {

constexpr size_t T = 130, HQ = 4, HKV = 2, D = 128, HK = 2, HV = 4, W = 32;

struct Tiny {  // the members nmg::Qwen35State reads, at a small size
    static constexpr size_t L = 4, CTX = 4096, Hkv = HKV, HEAD_DIM = D;
    static constexpr size_t KEY_HEADS = HK, VALUE_HEADS = HV, KEY_HEAD_DIM = D, VALUE_HEAD_DIM = D, CONV_WIDTH = 4;
    static constexpr bool is_recurrent(size_t layer) { return (layer + 1) % 4 != 0; }
};
enum class Kind { Local, Full };
struct TinyGemma {  // the members nmg::Gemma4Cache reads
    static constexpr size_t L = 6, CTX = 4096, Hkv = 1, LOCAL_HEAD_DIM = D, FULL_HEAD_DIM = D, LOCAL_WINDOW = W;
    static constexpr Kind attention_type(size_t layer) { return layer % 6 == 5 ? Kind::Full : Kind::Local; }
    static constexpr bool uses_shared_kv(size_t) { return false; }
};

std::string dir;

std::vector<float> load(const char* name, size_t n) {
    std::vector<float> h(n);
    FILE* f = std::fopen((dir + "/" + name).c_str(), "rb");
    if (!f || std::fread(h.data(), 4, n, f) != n) throw std::runtime_error(std::string("cannot read ") + name);
    std::fclose(f);
    return h;
}

void save(const char* name, const float* dptr, size_t n) {
    std::vector<float> h(n);
    if (cudaMemcpy(h.data(), dptr, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) throw std::runtime_error("copy back");
    FILE* f = std::fopen((dir + "/" + name).c_str(), "wb");
    if (!f || std::fwrite(h.data(), 4, n, f) != n) throw std::runtime_error(std::string("cannot write ") + name);
    std::fclose(f);
}

struct Dev {  // one device buffer of n floats, optionally filled from a file
    float* p = nullptr;
    explicit Dev(size_t n, const char* from = nullptr) {
        if (cudaMalloc(&p, n * 4) != cudaSuccess) throw std::runtime_error("cudaMalloc");
        if (from) {
            const auto h = load(from, n);
            if (cudaMemcpy(p, h.data(), n * 4, cudaMemcpyHostToDevice) != cudaSuccess) throw std::runtime_error("copy");
        }
    }
    ~Dev() { cudaFree(p); }
};

}  // namespace

int main(int argc, char** argv) {
    if (argc != 2) return 2;
    dir = argv[1];
    try {
        using nmg::Dtype;
        nmg::Qwen35State<Tiny> state(/*capacity*/ T + 1, Dtype::f32);
        // attention layer 3: append-then-reduce over T rows, then one decode row
        Dev q(T * HQ * D, "q.bin"), k(T * HKV * D, "k.bin"), v(T * HKV * D, "v.bin"), a(T * HQ * D);
        const float scale = 1.f / std::sqrt(float(D));
        nmg::append_attend<HQ>(state.attention(3), 0, k.p, v.p, Dtype::f32, q.p, Dtype::f32, T, &scale, a.p,
                               Dtype::f32, nullptr);
        Dev qd(HQ * D, "qd.bin"), kd(HKV * D, "kd.bin"), vd(HKV * D, "vd.bin"), ad(HQ * D);
        nmg::append_attend<HQ>(state.attention(3), T, kd.p, vd.p, Dtype::f32, qd.p, Dtype::f32, 1, &scale, ad.p,
                               Dtype::f32, nullptr);
        state.advance(T + 1);
        save("attn.bin", a.p, T * HQ * D);
        save("attn_decode.bin", ad.p, HQ * D);
        // recurrent layer 0: chunked delta-rule prefill from a zero state
        Dev dq(T * HK * D, "dq.bin"), dk(T * HK * D, "dk.bin"), dv(T * HV * D, "dv.bin"), g(T * HV, "g.bin"),
            b(T * HV, "b.bin"), o(T * HV * D);
        auto& rec = state.recurrent(0);
        rec.delta.prefill(HK, T, dq.p, dk.p, dv.p, g.p, b.p, o.p, 64, nullptr);
        save("delta.bin", o.p, T * HV * D);
        save("delta_state.bin", rec.delta.head(0), HV * D * D);
        // clear() forgets everything: the same prefill gives the same output
        state.clear(nullptr);
        if (state.tokens() != 0 || state.attention(3).size() != 0) throw std::logic_error("clear left state behind");
        rec.delta.prefill(HK, T, dq.p, dk.p, dv.p, g.p, b.p, o.p, 64, nullptr);
        save("delta_again.bin", o.p, T * HV * D);
        // a Gemma sliding-window layer (scale 1) whose batch is longer than the window
        nmg::Gemma4Cache<TinyGemma> gemma(/*capacity*/ T, /*local_capacity*/ T + W, Dtype::f32);
        Dev gq(T * D, "gq.bin"), gk(T * D, "gk.bin"), gv(T * D, "gv.bin"), ga(T * D);
        nmg::append_attend<1>(gemma.local(0), 0, gk.p, gv.p, Dtype::f32, gq.p, Dtype::f32, T, nullptr, ga.p,
                              Dtype::f32, nullptr);
        save("gemma_local.bin", ga.p, T * D);
        if (gemma.local(0).size() != W) throw std::logic_error("the ring does not hold the window");
        nmg::device_status(0, nullptr);
    } catch (const std::exception& e) {
        std::printf("FAIL: %s\n", e.what());
        return 1;
    }
    std::puts("PASS");
    return 0;
}
