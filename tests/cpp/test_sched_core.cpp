// Unit test of the continuous-batching policy (funasr-ggml_b200/csrc/sched_core.hpp)
// against a fake backend that keeps sequences and a page pool on the host and answers
// each output row with a token that depends only on (sequence content, position), so
// every stream's tokens must equal what the stream would produce decoded alone.
// Exit code 0 when every check passes.
#include "sched_core.hpp"

#include <cstdio>
#include <cstdlib>
#include <map>
#include <vector>

#define CHECK(c)                                                      \
    do {                                                              \
        if (!(c)) {                                                   \
            std::printf("CHECK failed: %s (line %d)\n", #c, __LINE__); \
            std::exit(1);                                             \
        }                                                             \
    } while (0)

struct Fake {
    int rows_cap = 64, seqs_cap = 6, H = 4;
    long pages = 40;
    long used_pages = 0, peak_pages = 0;
    int forwards = 0;
    struct S { bool open = false; int max_tokens = 0; std::vector<int> toks; long pages = 0; };
    std::vector<S> seqs = std::vector<S>(6);

    // token of position p in a sequence whose tokens so far are t: a hash of the content
    static int model(const std::vector<int>& t) {
        unsigned h = 2166136261u;
        for (int x : t) h = (h ^ (unsigned)x) * 16777619u;
        return (int)(h % 997);
    }
    int open(int max_tokens, int* seq) {
        for (int i = 0; i < seqs_cap; ++i)
            if (!seqs[i].open) {
                seqs[i] = S();
                seqs[i].open = true;
                seqs[i].max_tokens = max_tokens;
                *seq = i;
                return 0;
            }
        return -5;
    }
    int close(int seq) {
        CHECK(seqs[seq].open);
        used_pages -= seqs[seq].pages;
        seqs[seq] = S();
        return 0;
    }
    int forward(int n, const int* sq, const int* tok, const float* emb, int n_out, const int* out_rows, int* next) {
        ++forwards;
        CHECK(n >= 1 && n <= rows_cap);
        for (int i = 0; i < n; ++i) {
            S& s = seqs[sq[i]];
            CHECK(s.open);
            int t = tok[i];
            if (t == -1) {
                CHECK(emb != nullptr);
                t = 1000 + (int)emb[(size_t)i * H];   // embedding rows carry their id in element 0
                for (int k = 1; k < H; ++k) CHECK(emb[(size_t)i * H + k] == emb[(size_t)i * H] + k);
            }
            s.toks.push_back(t);
            CHECK((int)s.toks.size() <= s.max_tokens);
            const long need = ((long)s.toks.size() + 15) / 16;
            if (need > s.pages) {
                used_pages += need - s.pages;
                s.pages = need;
            }
            CHECK(used_pages <= pages);
            peak_pages = std::max(peak_pages, used_pages);
        }
        for (int k = 0; k < n_out; ++k) {
            CHECK(out_rows[k] >= 0 && out_rows[k] < n);
            // the content of the row's sequence up to and including that row
            const int seq = sq[out_rows[k]];
            int upto = 0;
            for (int i = 0; i <= out_rows[k]; ++i)
                if (sq[i] == seq) ++upto;
            const int have = (int)seqs[seq].toks.size();
            int cnt = 0;
            for (int i = 0; i < n; ++i)
                if (sq[i] == seq) ++cnt;
            std::vector<int> pre(seqs[seq].toks.begin(), seqs[seq].toks.begin() + (have - cnt + upto));
            next[k] = model(pre);
        }
        return 0;
    }
    long total_pages() const { return pages; }
    int max_rows() const { return rows_cap; }
    int max_seqs() const { return seqs_cap; }
    int hidden() const { return H; }
};

// the tokens a stream produces decoded alone
static std::vector<int> alone(const std::vector<int>& prompt, int max_new, int eos) {
    std::vector<int> t = prompt, out;
    for (int k = 0; k < max_new; ++k) {
        const int x = Fake::model(t);
        out.push_back(x);
        if (x == eos) break;
        t.push_back(x);
    }
    return out;
}

int main() {
    // 1. token prompts, more streams than slots and pages: FCFS admission, reservations
    {
        Fake be;
        fa::SchedConfig cfg;
        cfg.max_batch_rows = 64;
        cfg.prefill_chunk = 20;
        cfg.max_running = 8;
        fa::SchedCore<Fake> core(be, cfg);
        std::map<long, std::vector<int>> prompts;
        std::map<long, int> max_new;
        for (long tag = 0; tag < 15; ++tag) {
            std::vector<int> p((size_t)(5 + (tag * 37) % 90));
            for (size_t i = 0; i < p.size(); ++i) p[i] = (int)((tag * 131 + i * 7) % 900);
            prompts[tag] = p;
            max_new[tag] = 1 + (int)((tag * 53) % 60);
            CHECK(core.submit(tag, p.data(), nullptr, (int)p.size(), max_new[tag]) == 0);
        }
        // a stream larger than the whole pool is refused
        std::vector<int> huge(700, 1);
        CHECK(core.submit(99, huge.data(), nullptr, 700, 10) == -1);
        std::map<long, std::vector<int>> got;
        std::map<long, int> fin;
        std::vector<fa::SchedEvent> ev;
        int guard = 0;
        while (!core.idle()) {
            ev.clear();
            CHECK(core.step(ev) == 0);
            for (auto& e : ev) {
                CHECK(!fin.count(e.tag));
                got[e.tag].push_back(e.token);
                if (e.finished) fin[e.tag] = 1;
            }
            const fa::SchedStats st = core.stats();
            CHECK(st.reserved_pages <= st.total_pages);
            CHECK(st.running <= 6);
            CHECK(++guard < 10000);
        }
        for (long tag = 0; tag < 15; ++tag) {
            CHECK(fin.count(tag));
            CHECK(got[tag] == alone(prompts[tag], max_new[tag], -1));
        }
        CHECK(be.used_pages == 0);
        const fa::SchedStats st = core.stats();
        CHECK(st.finished == 15 && st.waiting == 0 && st.running == 0);
        std::printf("token prompts: %d forwards, peak %ld of %ld pages\n", be.forwards, be.peak_pages, be.pages);
    }
    // 2. embedding prompts mixed with token prompts, and an end-of-sequence id
    {
        Fake be;
        fa::SchedConfig cfg;
        cfg.max_batch_rows = 32;
        cfg.prefill_chunk = 16;
        cfg.max_running = 6;
        cfg.eos_id = 7;
        fa::SchedCore<Fake> core(be, cfg);
        std::map<long, std::vector<int>> prompts;
        for (long tag = 0; tag < 8; ++tag) {
            const int n = 3 + (int)((tag * 29) % 40);
            std::vector<int> ids((size_t)n);
            if (tag % 2) {
                std::vector<float> emb((size_t)n * 4);
                for (int i = 0; i < n; ++i) {
                    const int id = (int)((tag * 17 + i) % 50);
                    ids[(size_t)i] = 1000 + id;
                    for (int k = 0; k < 4; ++k) emb[(size_t)i * 4 + k] = (float)(id + k);
                }
                CHECK(core.submit(tag, nullptr, emb.data(), n, 40) == 0);
            } else {
                for (int i = 0; i < n; ++i) ids[(size_t)i] = (int)((tag * 61 + i * 3) % 900);
                CHECK(core.submit(tag, ids.data(), nullptr, n, 40) == 0);
            }
            prompts[tag] = ids;
        }
        std::map<long, std::vector<int>> got;
        std::vector<fa::SchedEvent> ev;
        while (!core.idle()) {
            ev.clear();
            CHECK(core.step(ev) == 0);
            for (auto& e : ev) got[e.tag].push_back(e.token);
        }
        for (long tag = 0; tag < 8; ++tag) CHECK(got[tag] == alone(prompts[tag], 40, 7));
        std::printf("mixed prompts with eos: %d forwards\n", be.forwards);
    }
    std::printf("OK\n");
    return 0;
}
