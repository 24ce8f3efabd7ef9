// Test harness for llm-inference-diy_b200/csrc/batch_sched.h: runs the continuous-batching
// scheduler against a fake model whose next token depends only on (token, position), and
// prints every callback so that tests/test_sched_cpu.py can check it.  Input (stdin):
//   slots max_len max_new stop_on_eos vocab
//   one request per line (space-separated ids; an empty line is an empty request), then "end"
// Output lines: "P slot n" (prefill), "S B" (decode step), "E r t" (emit), "D r why" (done), "RC rc".
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "batch_sched.h"

// next token of the fake model; a stop id now and then
static int fake_next(int t, int p) {
    if ((t + 3 * p) % 23 == 0) return 151645;
    return (t * 31 + p * 7 + 3) % 997;
}

int main() {
    llmdiy::SchedConfig c{};
    int stop = 0;
    std::cin >> c.slots >> c.max_len >> c.max_new >> stop >> c.vocab;
    c.stop_on_eos = stop != 0;
    std::string line;
    std::getline(std::cin, line);
    std::vector<std::vector<int>> reqs;
    while (std::getline(std::cin, line) && line != "end") {
        std::istringstream is(line);
        std::vector<int> p;
        int v;
        while (is >> v) p.push_back(v);
        reqs.push_back(p);
    }
    const int fail_after = std::getenv("FAIL_AFTER") ? std::atoi(std::getenv("FAIL_AFTER")) : -1;
    int steps = 0;
    const int rc = llmdiy::run_continuous_batch(
        c, reqs,
        [&](int s, const int*, int n) {
            std::cout << "P " << s << " " << n << "\n";
            return 0;
        },
        [&](int B, const int* t, const int* p, int* out) {
            if (steps == fail_after) return 7;
            ++steps;
            std::cout << "S " << B;
            for (int i = 0; i < B; ++i) std::cout << " " << t[i] << ":" << p[i];
            std::cout << "\n";
            for (int i = 0; i < B; ++i) out[i] = fake_next(t[i], p[i]);
            return 0;
        },
        [&](int r, int t) { std::cout << "E " << r << " " << t << "\n"; },
        [&](int r, int why) { std::cout << "D " << r << " " << why << "\n"; });
    std::cout << "RC " << rc << "\n";
    return 0;
}
