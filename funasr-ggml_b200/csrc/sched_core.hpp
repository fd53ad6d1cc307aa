// Continuous-batching scheduler for many utterance streams on one GPU: the policy,
// independent of the device so that it can be tested against a fake backend.
//
// The reference decodes one utterance at a time (pipeline/pipeline.cpp:434-451): a
// prefill, then one forward per token, its KV cache cleared per utterance
// (compute/gpu_context.hpp:116-122). Here every call to step() runs ONE forward over a
// batch of rows drawn from all live streams:
//   1. admission, first come first served: a waiting stream is admitted when a
//      sequence slot is free and the pool can hold its whole lifetime (prompt + max
//      new tokens, in pages); its pages are reserved, so a running stream never
//      meets an exhausted pool and nothing is ever preempted;
//   2. batch: one decode row per stream that has finished its prompt (it feeds the
//      stream's last token), then prompt rows of streams still in prefill, up to
//      `prefill_chunk` rows per stream, in admission order, until `max_batch_rows`;
//   3. outputs only for rows that produce a token: decode rows and the last prompt
//      row of a stream (its first generated token);
//   4. a stream finishes at max_new tokens or at the end-of-sequence id; its
//      sequence is closed, which returns its pages to the pool, and its reservation
//      is released.
// Backend interface (see scheduler.cpp for the device one):
//   int  open(int max_tokens, int* seq)        0 or a negative error
//   int  close(int seq)
//   int  forward(n_rows, seq_ids, token_ids (-1: row from embeds), embeds | nullptr,
//                n_out, out_rows, next_ids)
//   long total_pages(); int max_rows(); int max_seqs(); int hidden();
#pragma once

#include <algorithm>
#include <cstdint>
#include <deque>
#include <memory>
#include <string>
#include <vector>

namespace fa {

struct SchedConfig {
    int max_batch_rows = 512;   // rows per forward (decode rows + prompt rows)
    int prefill_chunk = 512;    // prompt rows of one stream per forward
    int max_running = 256;      // streams admitted at once
    int eos_id = -1;            // end-of-sequence token; -1: generate exactly max_new tokens
};

struct SchedEvent {
    int64_t tag;     // the caller's id of the stream
    int token;       // generated token, or -1 for a stream that failed
    int finished;    // 1 on the stream's last event
};

struct SchedStats {
    long steps = 0;
    long rows = 0;              // rows run through the decoder
    long prompt_rows = 0;
    long tokens = 0;            // tokens generated
    long finished = 0;
    int waiting = 0;
    int running = 0;
    long reserved_pages = 0;
    long total_pages = 0;
};

template <typename Backend>
class SchedCore {
public:
    SchedCore(Backend& b, const SchedConfig& c) : be_(b), cfg_(c) {
        cfg_.max_batch_rows = std::max(1, std::min(cfg_.max_batch_rows, be_.max_rows()));
        cfg_.prefill_chunk = std::max(1, std::min(cfg_.prefill_chunk, cfg_.max_batch_rows));
        cfg_.max_running = std::max(1, std::min(cfg_.max_running, be_.max_seqs()));
    }

    // Queue a stream. Prompt as token ids or as embedding rows [n_prompt][hidden]
    // (exactly one). Returns 0, or -1 when the stream could never fit the pool.
    int submit(int64_t tag, const int* ids, const float* embeds, int n_prompt, int max_new) {
        if (n_prompt <= 0 || max_new <= 0 || (ids == nullptr) == (embeds == nullptr)) return -1;
        auto s = std::make_unique<Stream>();
        s->tag = tag;
        s->n_prompt = n_prompt;
        s->max_new = max_new;
        if (ids) s->ids.assign(ids, ids + n_prompt);
        else s->emb.assign(embeds, embeds + (size_t)n_prompt * be_.hidden());
        s->pages = pages_for(n_prompt + max_new);
        if (s->pages > be_.total_pages()) return -1;
        waiting_.push_back(std::move(s));
        return 0;
    }

    bool idle() const { return waiting_.empty() && running_.empty(); }

    // One scheduling round and one forward. Appends events; returns 0 or the
    // backend's error (the streams of a failed forward are failed and retired).
    int step(std::vector<SchedEvent>& events) {
        admit();
        if (running_.empty()) return 0;
        rows_seq_.clear();
        rows_tok_.clear();
        rows_emb_.clear();
        out_rows_.clear();
        out_owner_.clear();
        bool any_emb = false;
        const int H = be_.hidden();
        // decode rows
        for (auto& s : running_) {
            if ((int)rows_seq_.size() >= cfg_.max_batch_rows) break;
            if (s->prefilled < s->n_prompt || s->done) continue;
            out_rows_.push_back((int)rows_seq_.size());
            out_owner_.push_back(s.get());
            rows_seq_.push_back(s->seq);
            rows_tok_.push_back(s->last);
        }
        // prompt rows
        const size_t n_decode = rows_seq_.size();
        std::vector<std::pair<Stream*, int>> chunks;
        for (auto& s : running_) {
            const int room = cfg_.max_batch_rows - (int)rows_seq_.size();
            if (room <= 0) break;
            if (s->prefilled >= s->n_prompt) continue;
            const int n = std::min({cfg_.prefill_chunk, s->n_prompt - s->prefilled, room});
            for (int k = 0; k < n; ++k) {
                rows_seq_.push_back(s->seq);
                if (s->ids.empty()) {
                    rows_tok_.push_back(-1);
                    any_emb = true;
                } else {
                    rows_tok_.push_back(s->ids[(size_t)s->prefilled + k]);
                }
            }
            if (s->prefilled + n == s->n_prompt) {
                out_rows_.push_back((int)rows_seq_.size() - 1);
                out_owner_.push_back(s.get());
            }
            chunks.push_back({s.get(), n});
        }
        if (any_emb) {
            // embedding rows of prompts given as embeddings; the other rows use token ids
            rows_emb_.assign(rows_seq_.size() * (size_t)H, 0.0f);
            size_t pos = n_decode;
            for (auto& c : chunks) {
                const Stream* s = c.first;
                if (!s->emb.empty())
                    std::copy(s->emb.begin() + (size_t)s->prefilled * H,
                              s->emb.begin() + (size_t)(s->prefilled + c.second) * H, rows_emb_.begin() + pos * H);
                pos += (size_t)c.second;
            }
        }
        next_.assign(out_rows_.size(), 0);
        const int rc = be_.forward((int)rows_seq_.size(), rows_seq_.data(), rows_tok_.data(),
                                   any_emb ? rows_emb_.data() : nullptr, (int)out_rows_.size(), out_rows_.data(),
                                   next_.data());
        ++stats_.steps;
        if (rc != 0) {
            for (auto& s : running_) {
                events.push_back({s->tag, -1, 1});
                s->done = true;
            }
            retire();
            return rc;
        }
        stats_.rows += (long)rows_seq_.size();
        for (auto& c : chunks) {
            c.first->prefilled += c.second;
            stats_.prompt_rows += c.second;
        }
        for (size_t k = 0; k < out_rows_.size(); ++k) {
            Stream* s = out_owner_[k];
            const int tok = next_[k];
            ++s->generated;
            ++stats_.tokens;
            s->last = tok;
            const bool fin = s->generated >= s->max_new || (cfg_.eos_id >= 0 && tok == cfg_.eos_id);
            events.push_back({s->tag, tok, fin ? 1 : 0});
            if (fin) s->done = true;
        }
        retire();
        return 0;
    }

    SchedStats stats() const {
        SchedStats s = stats_;
        s.waiting = (int)waiting_.size();
        s.running = (int)running_.size();
        s.reserved_pages = reserved_;
        s.total_pages = be_.total_pages();
        return s;
    }

private:
    struct Stream {
        int64_t tag = 0;
        std::vector<int> ids;
        std::vector<float> emb;
        int n_prompt = 0, max_new = 0;
        int seq = -1;
        int prefilled = 0;
        int generated = 0;
        int last = -1;
        long pages = 0;
        bool done = false;
    };

    static long pages_for(int tokens) { return (tokens + 15) / 16; }

    void admit() {
        while (!waiting_.empty() && (int)running_.size() < cfg_.max_running) {
            Stream& s = *waiting_.front();
            if (reserved_ + s.pages > be_.total_pages()) break;
            int seq = -1;
            if (be_.open(s.n_prompt + s.max_new, &seq) != 0) break;
            s.seq = seq;
            reserved_ += s.pages;
            running_.push_back(std::move(waiting_.front()));
            waiting_.pop_front();
        }
    }

    void retire() {
        for (size_t i = 0; i < running_.size();) {
            if (running_[i]->done) {
                be_.close(running_[i]->seq);
                reserved_ -= running_[i]->pages;
                ++stats_.finished;
                running_.erase(running_.begin() + (long)i);
            } else {
                ++i;
            }
        }
    }

    Backend& be_;
    SchedConfig cfg_;
    std::deque<std::unique_ptr<Stream>> waiting_;
    std::vector<std::unique_ptr<Stream>> running_;
    long reserved_ = 0;
    SchedStats stats_;
    std::vector<int> rows_seq_, rows_tok_, out_rows_, next_;
    std::vector<Stream*> out_owner_;
    std::vector<float> rows_emb_;
};

}  // namespace fa
