// batch_sched.h — continuous (iteration-level) batching of independent greedy
// requests over the slots of a llmdiy_batch (include/llmdiy_batch.h).
//
// The reference serves one sequence per turn (framework_src/qwen_infer.cu:786-818:
// prefill prompt[0..n-2], then step() from prompt[n-1] at position n-1 until a stop
// id or 512 tokens).  Here every request follows the same per-sequence rule, but up
// to `slots` requests decode together: each iteration runs one batched step for the
// active slots, retires the requests that finished, and admits waiting requests into
// the freed slots (prefilled before the next step).  Host-only logic; the GPU work is
// behind the prefill/decode callbacks, so the scheduler can be exercised without a GPU.
#pragma once
#include <cstddef>
#include <deque>
#include <vector>

namespace llmdiy {

struct SchedConfig {
    int slots;         // sequences decoded together (<= the batch's max_batch)
    int max_len;       // positions per slot (the batch's max_len)
    int max_new;       // tokens generated per request at most (the reference driver's 512)
    bool stop_on_eos;  // stop at the stop ids (151645, 151643), which are not emitted
    int vocab;         // valid token ids are [0, vocab)
};

enum SchedDone { DONE_STOP = 0, DONE_LENGTH = 1, DONE_REJECTED = 2 };

// Runs every request to completion.  Callbacks:
//   int prefill(int slot, const int* tokens, int n)      prompt rows 0..n-1 of a slot (n >= 1)
//   int decode(int B, const int* tok, const int* pos, int* out)   one step of slots 0..B-1
//   void emit(int request, int token)                     a generated token, in order
//   void done(int request, int why)                       a SchedDone value
// B is the highest occupied slot + 1 (it only grows while requests wait); slots below
// B that hold no request decode a dummy token at position 0 (their row 0 is free).
// A callback's non-zero return stops the run and is returned; requests not yet
// finished get no done() call then.
template <class Prefill, class Decode, class Emit, class Done>
int run_continuous_batch(const SchedConfig& cfg, const std::vector<std::vector<int>>& requests, Prefill&& prefill,
                         Decode&& decode, Emit&& emit, Done&& done) {
    struct Slot {
        int req = -1;   // request in this slot, -1 = free
        int token = 0;  // token fed to the next step
        int pos = 0;    // its position
        int made = 0;   // tokens generated so far
        int limit = 0;  // tokens this request may generate
    };
    std::vector<Slot> slot((size_t)cfg.slots);
    std::deque<int> waiting;
    for (int r = 0; r < (int)requests.size(); ++r) waiting.push_back(r);
    std::vector<int> tok((size_t)cfg.slots), pos((size_t)cfg.slots), out((size_t)cfg.slots);
    int active = 0, B = 0;
    while (!waiting.empty() || active > 0) {
        // admit waiting requests into free slots, lowest slot first
        for (int s = 0; s < cfg.slots && !waiting.empty(); ++s) {
            if (slot[(size_t)s].req >= 0) continue;
            while (!waiting.empty()) {
                const int r = waiting.front();
                waiting.pop_front();
                const std::vector<int>& p = requests[(size_t)r];
                const int n = (int)p.size();
                bool ok = n >= 1 && n <= cfg.max_len;
                for (int i = 0; ok && i < n; ++i) ok = p[(size_t)i] >= 0 && p[(size_t)i] < cfg.vocab;
                if (!ok) {
                    done(r, DONE_REJECTED);
                    continue;
                }
                if (n > 1) {
                    const int rc = prefill(s, p.data(), n - 1);
                    if (rc) return rc;
                }
                Slot& q = slot[(size_t)s];
                q.req = r;
                q.token = p[(size_t)n - 1];
                q.pos = n - 1;
                q.made = 0;
                // steps run at positions n-1 .. max_len-1, one token each
                q.limit = cfg.max_new < cfg.max_len - n + 1 ? cfg.max_new : cfg.max_len - n + 1;
                ++active;
                if (s + 1 > B) B = s + 1;
                break;
            }
        }
        if (active == 0) break;
        for (int s = 0; s < B; ++s) {
            const Slot& q = slot[(size_t)s];
            tok[(size_t)s] = q.req >= 0 ? q.token : 0;
            pos[(size_t)s] = q.req >= 0 ? q.pos : 0;
        }
        const int rc = decode(B, tok.data(), pos.data(), out.data());
        if (rc) return rc;
        for (int s = 0; s < B; ++s) {
            Slot& q = slot[(size_t)s];
            if (q.req < 0) continue;
            const int t = out[(size_t)s];
            ++q.made;
            const bool stop = cfg.stop_on_eos && (t == 151645 || t == 151643);
            if (!stop) emit(q.req, t);
            if (stop || q.made >= q.limit) {
                done(q.req, stop ? DONE_STOP : DONE_LENGTH);
                q.req = -1;
                --active;
                continue;
            }
            q.token = t;
            ++q.pos;
        }
        // B stays at its high-water mark while requests wait (freed slots are refilled at once);
        // with none waiting it shrinks to the highest occupied slot, so it changes (and the
        // batch re-captures its step graph) at most once per retired slot
        if (waiting.empty())
            while (B > 0 && slot[(size_t)B - 1].req < 0) --B;
    }
    return 0;
}

}  // namespace llmdiy
