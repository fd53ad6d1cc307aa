// Decoder test through the C++ host API (include/funasr_b200.hpp), written the way the
// reference's own GPU tests drive its classes (test/test_gpu.cpp, test/test_llm.cpp):
// load a model file, warm up, prefill, greedy decode with GPURunner::argmax, then
// check the cache bookkeeping.
//
// Build (tests/test_cpp_api.py does this), from the repository root:
//   g++ -std=c++17 -O2 -I include tests/cpp/test_decoder_api.cpp -L funasr-ggml_b200
//       -lfunasr_dec -Wl,-rpath,<absolute path of funasr-ggml_b200> -o test_decoder_api
// Run:
//   ./test_decoder_api <model.gguf> <prompt.f32> <n_prompt> <n_new> <out.bin>
// prompt.f32 holds n_prompt rows of embedding_length f32 (the adaptor's output in the
// full pipeline). out.bin receives, in order: n_new int32 greedy ids, vocab f32 logits of
// the last step, n_past x kv_dim u16 layer-0 K, the same for V, then the same ids again
// from the utterance decoded by BatchDecoder on a second sequence (n_new int32) and by the
// Scheduler (n_new int32).
// Exit codes: 0 ok, 1 usage / input, 2 GPU init failed, 3 forward failed, 4 check failed.
#include "funasr_b200.hpp"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

using namespace funasr_b200;

#define CHECK(cond)                                                  \
    do {                                                             \
        if (!(cond)) {                                               \
            std::printf("CHECK failed: %s (line %d)\n", #cond, __LINE__); \
            return 4;                                                \
        }                                                            \
    } while (0)

int main(int argc, char** argv) {
    if (argc < 6) {
        std::printf("Usage: %s <model.gguf> <prompt.f32> <n_prompt> <n_new> <out.bin>\n", argv[0]);
        return 1;
    }
    const std::string model = argv[1];
    const int n_prompt = std::atoi(argv[3]), n_new = std::atoi(argv[4]);

    std::printf("========================================\n");
    std::printf("  Decoder test through funasr_b200.hpp\n");
    std::printf("========================================\n");

    // 1. GPU context from the model file (two sequence slots: the context's own + one batch stream)
    GPUContext ctx;
    PoolOptions opt;
    opt.max_seqs = 2;
    opt.max_rows = 64;
    if (!ctx.init(model, 512, 0, opt)) {
        std::printf("GPU init failed: %s\n", ctx.last_error().c_str());
        return 2;
    }
    const LLMConfig& cfg = ctx.config();
    std::printf("model: %d layers, hidden %d, vocab %d, kv_dim %d\n", cfg.block_count, cfg.embedding_length,
                cfg.vocab_size, cfg.kv_dim());

    std::vector<float> prompt((size_t)n_prompt * cfg.embedding_length);
    {
        std::ifstream f(argv[2], std::ios::binary);
        if (!f.read(reinterpret_cast<char*>(prompt.data()), (std::streamsize)(prompt.size() * sizeof(float)))) {
            std::printf("cannot read %s\n", argv[2]);
            return 1;
        }
    }

    // 2. warmup, which must leave the cache empty
    GPURunner runner(ctx);
    if (!runner.warmup(32, 64)) return 3;
    CHECK(runner.is_warmed_up());
    CHECK(ctx.kv_cache().n_past == 0);

    // 3. prefill, then greedy decode exactly as the reference's loop (EOS ignored)
    std::vector<float> logits;
    if (!runner.forward(prompt.data(), n_prompt, 0, logits)) return 3;
    CHECK((int)logits.size() == cfg.vocab_size);
    CHECK(ctx.kv_cache().n_past == n_prompt);
    CHECK(GPURunner::argmax(logits) == runner.last_next_id());
    std::vector<int> ids;
    for (int step = 0; step < n_new; ++step) {
        const int next = GPURunner::argmax(logits);
        ids.push_back(next);
        if (!runner.forward_tokens(&next, 1, ctx.kv_cache().n_past, logits)) return 3;
        CHECK(GPURunner::argmax(logits) == runner.last_next_id());
    }
    CHECK(ctx.kv_cache().n_past == n_prompt + n_new);
    for (int i = 0; i < n_new; ++i) std::printf("%d ", ids[i]);
    std::printf("\n");

    // 4. the layer-0 cache in the reference's [n_past][kv_dim] order
    std::vector<uint16_t> k0, v0;
    CHECK(KVCache::read_sequence_layer(ctx, ctx.seq(), ctx.kv_cache().n_past, 0, k0, v0));
    CHECK(k0.size() == (size_t)ctx.kv_cache().n_past * cfg.kv_dim());

    // 5. rewinding: re-running the last step from n_past - 1 gives the same logits
    {
        const int last = ids.back();
        std::vector<float> again;
        if (!runner.forward_tokens(&last, 1, ctx.kv_cache().n_past - 1, again)) return 3;
        CHECK(again == logits);
    }

    // 5b. the reference's KVCache step contract on a cache of its own: set_pending per
    //     layer, commit at n_past, read back through k_tensor() / v_tensor(); a rewind
    //     commit overwrites; a layer with nothing pending reads zeros
    {
        KVCache kv;
        CHECK(kv.init(ctx, 64));
        const int L = kv.n_layers(), kvd = kv.kv_dim(), T = 20;
        std::vector<std::vector<float>> kf((size_t)L), vf((size_t)L);
        for (int l = 0; l < L; ++l) {
            kf[(size_t)l].resize((size_t)T * kvd);
            vf[(size_t)l].resize((size_t)T * kvd);
            for (size_t i = 0; i < kf[(size_t)l].size(); ++i) {
                kf[(size_t)l][i] = std::sin(0.001f * (float)(i + 7 * l)) * 3.0f;
                vf[(size_t)l][i] = std::cos(0.002f * (float)(i + 5 * l)) * 0.01f;
            }
            kv.set_pending(l, kf[(size_t)l].data(), vf[(size_t)l].data());
        }
        CHECK(kv.commit(0, T));
        CHECK(kv.n_past() == T);
        for (int l = 0; l < L; ++l) {
            std::vector<uint16_t> kr, vr;
            CHECK(kv.k_tensor().read(l, kr) && kv.v_tensor().read(l, vr));
            CHECK(kr.size() == (size_t)T * kvd && vr.size() == (size_t)T * kvd);
            for (size_t i = 0; i < kr.size(); ++i) {
                CHECK(kr[i] == f32_to_f16_bits(kf[(size_t)l][i]));
                CHECK(vr[i] == f32_to_f16_bits(vf[(size_t)l][i]));
            }
        }
        // rewind to 10 and commit 3 new tokens for layer 0 only
        std::vector<float> k3((size_t)3 * kvd, 1.5f), v3((size_t)3 * kvd, -2.0f);
        kv.set_pending(0, k3.data(), v3.data());
        CHECK(kv.commit(10, 3));
        CHECK(kv.n_past() == 13);
        std::vector<uint16_t> kr0, kr1;
        CHECK(kv.k_tensor().read(0, kr0) && kv.k_tensor().read(L - 1, kr1));
        CHECK(kr0[(size_t)5 * kvd] == f32_to_f16_bits(kf[0][(size_t)5 * kvd]));
        CHECK(kr0[(size_t)11 * kvd] == f32_to_f16_bits(1.5f));
        CHECK(kr1[(size_t)11 * kvd] == 0);
        CHECK(!kv.commit(20, 1));   // past the cached length
        kv.free();
    }

    // 6. the same utterance as a second stream through BatchDecoder
    BatchDecoder batch(ctx);
    const int s = batch.open(512);
    CHECK(s >= 0);
    int tok = -1;
    CHECK(batch.prefill(s, prompt.data(), n_prompt, &tok));
    std::vector<int> ids2;
    for (int step = 0; step < n_new; ++step) {
        ids2.push_back(tok);
        std::vector<int> nx;
        CHECK(batch.step({s}, {tok}, nx));
        tok = nx[0];
    }
    int len = 0;
    fa_seq_length(ctx.handle(), s, &len);
    CHECK(len == n_prompt + n_new);
    CHECK(batch.close(s));

    // 7. the same utterance through the scheduler, one prompt chunk (graphs off: every
    //    scheduled step has its own shape)
    std::vector<int> ids3;
    {
        fa_set_graphs(ctx.handle(), 0);
        Scheduler::Config sc;
        sc.max_batch_rows = 64;
        sc.prefill_chunk = 64;
        sc.max_running = 1;
        sc.eos_id = -1;
        Scheduler sch(ctx, sc);
        CHECK(sch.ok());
        CHECK(sch.submit_embeds(7, prompt.data(), n_prompt, n_new));
        std::vector<fa_sched_event> ev;
        int guard = 0;
        while (!sch.idle()) {
            CHECK(sch.step(ev));
            for (const auto& e : ev) {
                CHECK(e.tag == 7 && e.token >= 0);
                ids3.push_back(e.token);
            }
            CHECK(++guard < 10000);
        }
        CHECK((int)ids3.size() == n_new);
        CHECK(sch.stats().finished == 1);
        fa_set_graphs(ctx.handle(), 1);
    }

    // 8. clear_kv_cache empties the context's own sequence
    ctx.clear_kv_cache();
    CHECK(ctx.kv_cache().n_past == 0);

    std::ofstream out(argv[5], std::ios::binary);
    out.write(reinterpret_cast<const char*>(ids.data()), (std::streamsize)(ids.size() * sizeof(int)));
    out.write(reinterpret_cast<const char*>(logits.data()), (std::streamsize)(logits.size() * sizeof(float)));
    out.write(reinterpret_cast<const char*>(k0.data()), (std::streamsize)(k0.size() * 2));
    out.write(reinterpret_cast<const char*>(v0.data()), (std::streamsize)(v0.size() * 2));
    out.write(reinterpret_cast<const char*>(ids2.data()), (std::streamsize)(ids2.size() * sizeof(int)));
    out.write(reinterpret_cast<const char*>(ids3.data()), (std::streamsize)(ids3.size() * sizeof(int)));
    std::printf("OK\n");
    return 0;
}
