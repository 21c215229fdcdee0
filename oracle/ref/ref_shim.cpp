// ref_shim.cpp — C entry points around the reference's own model code.
//
// TEST INFRASTRUCTURE: linked only into oracle/_ref/libref.so together with
// the reference's unchanged sources (backend, parser, models, adapter loader),
// compiled where they lie.  Used on the GPU box to produce golden logits that
// pin the CPU oracle (tests/golden/make_golden.py).  The product never loads it.
#include <tensor/adapter/adapter_loader.hpp>
#include <tensor/backend/ops.hpp>
#include <tensor/inference/sampling/greedy.hpp>
#include <tensor/inference/sampling/top_p.hpp>
#include <tensor/models/gemma/gemma_model.hpp>
#include <tensor/models/llama/llama_model.hpp>
#include <tensor/models/mistral/mistral_model.hpp>
#include <tensor/models/qwen/qwen_adapter_model.hpp>
#include <tensor/models/qwen/qwen_model.hpp>
#include <tensor/parser/config.hpp>
#include <tensor/parser/weight_map.hpp>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <exception>
#include <thread>
#include <vector>

namespace ops = tensor::backend::ops;

namespace {

// logits [seq, vocab] bf16 -> fp32 last row (the row Generator samples from)
void last_row(const tensor::backend::Tensor& lg, float* out, int vocab) {
    auto f = ops::cast(lg, tensor::backend::DType::F32);
    std::vector<float> h = f.to_host_f32();
    std::memcpy(out, h.data() + (h.size() - (size_t)vocab), (size_t)vocab * 4);
}

template <class M>
void run(M& model, const int32_t* prompt, int n_prompt, const int32_t* feed, int n_steps, int max_seq, float* logits,
         int vocab) {
    auto cache = model.make_cache((std::size_t)max_seq);
    std::vector<int32_t> ids(prompt, prompt + n_prompt);
    auto lg = model.forward(ids, cache);
    last_row(lg, logits, vocab);
    for (int i = 0; i < n_steps; ++i) {
        lg = model.forward(std::vector<int32_t>{feed[i]}, cache);
        last_row(lg, logits + (size_t)(i + 1) * vocab, vocab);
    }
}

}  // namespace

// arch: 0 llama, 1 qwen2, 2 gemma, 3 mistral; adapter_dir (qwen2 only) may be NULL.
// logits: (1 + n_steps) x vocab fp32 — the prompt's last row, then one row per fed token.
extern "C" int ref_run(const char* model_dir, int arch, const char* adapter_dir, const int32_t* prompt, int n_prompt,
                       const int32_t* feed, int n_steps, int max_seq, float* logits, int vocab, char* err,
                       int err_len) {
    try {
        const auto dev = tensor::backend::Device::cuda(0);
        auto wm = tensor::parser::WeightMap::open(model_dir);
        auto cfg = tensor::parser::ModelConfig::from_dir(model_dir);
        switch (arch) {
            case 0: {
                auto m = tensor::models::llama::LlamaModel::load(wm, cfg, dev);
                run(m, prompt, n_prompt, feed, n_steps, max_seq, logits, vocab);
                break;
            }
            case 1: {
                auto m = tensor::models::qwen::QwenModel::load(wm, cfg, dev);
                if (adapter_dir) {
                    auto aw = tensor::adapter::AdapterLoader::load(adapter_dir, "qwen2", cfg.num_hidden_layers(), dev);
                    tensor::models::qwen::QwenAdapterModel am(std::move(m), std::move(aw));
                    run(am, prompt, n_prompt, feed, n_steps, max_seq, logits, vocab);
                } else {
                    run(m, prompt, n_prompt, feed, n_steps, max_seq, logits, vocab);
                }
                break;
            }
            case 2: {
                auto m = tensor::models::gemma::GemmaModel::load(wm, cfg, dev);
                run(m, prompt, n_prompt, feed, n_steps, max_seq, logits, vocab);
                break;
            }
            case 3: {
                auto m = tensor::models::mistral::MistralModel::load(wm, model_dir, dev);
                run(m, prompt, n_prompt, feed, n_steps, max_seq, logits, vocab);
                break;
            }
            default: std::snprintf(err, err_len, "unknown arch %d", arch); return 2;
        }
        return 0;
    } catch (const std::exception& e) {
        std::snprintf(err, err_len, "%s", e.what());
        return 1;
    }
}

// Decode-step timing of the reference's own CUDA path on this GPU (Llama
// model files, llama_model.cpp:210-238): the prompt in one forward call, then
// n_warm + n_steps single-token steps, each followed by the reference's own
// Greedy::sample (greedy.cpp:11-36, as Generator::generate does per token,
// generator.cpp:24-84), its id fed back.  ms_per_step: wall time of the last
// n_steps steps over n_steps; the reference's ops synchronise the device.
extern "C" int ref_time_decode(const char* model_dir, const int32_t* prompt, int n_prompt, int n_warm, int n_steps,
                               int max_seq, double* ms_per_step, int32_t* last_id, char* err, int err_len) {
    try {
        const auto dev = tensor::backend::Device::cuda(0);
        auto wm = tensor::parser::WeightMap::open(model_dir);
        auto cfg = tensor::parser::ModelConfig::from_dir(model_dir);
        auto m = tensor::models::llama::LlamaModel::load(wm, cfg, dev);
        auto cache = m.make_cache((std::size_t)max_seq);
        std::vector<int32_t> ids(prompt, prompt + n_prompt);
        auto lg = m.forward(ids, cache);
        const int vocab = (int)m.vocab_size();
        int32_t tok = tensor::inference::sampling::Greedy{}.sample(lg);
        auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < n_warm + n_steps; ++i) {
            if (i == n_warm) t0 = std::chrono::steady_clock::now();
            lg = m.forward(std::vector<int32_t>{((tok % vocab) + vocab) % vocab}, cache);
            tok = tensor::inference::sampling::Greedy{}.sample(lg);
        }
        const auto t1 = std::chrono::steady_clock::now();
        *ms_per_step = std::chrono::duration<double, std::milli>(t1 - t0).count() / std::max(1, n_steps);
        *last_id = tok;
        return 0;
    } catch (const std::exception& e) {
        std::snprintf(err, err_len, "%s", e.what());
        return 1;
    }
}

// The reference's samplers (src/inference/sampling/greedy.cpp, top_p.cpp) on a
// host tensor of fp32 logits [rows, vocab]; they read the last row.
// kind: 0 Greedy, 1 TopP(temperature, p), 2 TopK(temperature, k); seeded = 0
// leaves the seed unset (std::random_device).  out[i] = the i-th of n_draws
// sample() calls, all made on one fresh thread: TopP's engine is a
// thread_local seeded at its first call on a thread (top_p.cpp:84), so a new
// thread restarts the sequence.  Needs no GPU.
extern "C" int ref_sample(const float* logits, int rows, int vocab, int kind, float temperature, float p, uint32_t k,
                          int seeded, uint64_t seed, int n_draws, int32_t* out, char* err, int err_len) {
    int rc = 0;
    std::thread th([&] {
        try {
            namespace smp = tensor::inference::sampling;
            tensor::core::TensorView view;
            view.data = logits;
            view.dtype = tensor::backend::DType::F32;
            view.shape = tensor::backend::Shape{(std::size_t)rows, (std::size_t)vocab};
            auto t = tensor::backend::Tensor::from_view(view, tensor::backend::Device::cpu());
            smp::TopP tp;
            tp.temperature = temperature;
            tp.p = p;
            smp::TopK tk;
            tk.temperature = temperature;
            tk.k = k;
            if (seeded) tp.seed = tk.seed = seed;
            for (int i = 0; i < n_draws; ++i) {
                switch (kind) {
                    case 0: out[i] = smp::Greedy{}.sample(t); break;
                    case 1: out[i] = tp.sample(t); break;
                    case 2: out[i] = tk.sample(t); break;
                    default: std::snprintf(err, err_len, "unknown sampler %d", kind); rc = 2; return;
                }
            }
        } catch (const std::exception& e) {
            std::snprintf(err, err_len, "%s", e.what());
            rc = 1;
        }
    });
    th.join();
    return rc;
}
