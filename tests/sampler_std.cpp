// The daemon's token draw written against the C++ standard library itself
// (std::partial_sort, std::exp on float, std::discrete_distribution,
// std::mt19937), the arithmetic of sample_token_cpp and of the text rule in
// utkarshyadav009/bmo_jetson src/bmo_daemon.cpp:147-175 and :755-762.  The
// CPU tests compile it with the host compiler to pin the Python restatement
// (tests/sampler.py) to libstdc++'s behaviour.  TEST INFRASTRUCTURE.
//
// stdin:  seed n_cases, then per case: n temp top_k rule, then n logits
//         (rule 0: one draw; rule 1: the daemon's text rule with sampling on)
// stdout: one token per case, all cases drawing from one generator.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <random>
#include <utility>
#include <vector>

static int draw(const std::vector<float> &logits, float temp, int top_k, std::mt19937 &rng) {
    const int n = static_cast<int>(logits.size());
    if (top_k <= 0 || temp <= 1e-4f) return static_cast<int>(std::max_element(logits.begin(), logits.end()) - logits.begin());
    std::vector<std::pair<float, int>> v(n);
    for (int i = 0; i < n; ++i) v[i] = {logits[i], i};
    const int k = std::min(top_k, n);
    std::partial_sort(v.begin(), v.begin() + k, v.end(),
                      [](const std::pair<float, int> &a, const std::pair<float, int> &b) { return a.first > b.first; });
    const float max_l = v[0].first / temp;
    std::vector<float> p(k);
    float sum = 0.0f;
    for (int i = 0; i < k; ++i) {
        p[i] = std::exp(v[i].first / temp - max_l);
        sum += p[i];
    }
    if (sum <= 0.0f || std::isnan(sum)) return v[0].second;
    std::discrete_distribution<int> dist(p.begin(), p.end());
    return v[dist(rng)].second;
}

int main() {
    unsigned seed = 0;
    int cases = 0;
    if (std::scanf("%u %d", &seed, &cases) != 2) return 1;
    std::mt19937 rng(seed);
    for (int c = 0; c < cases; ++c) {
        int n = 0, top_k = 0, rule = 0;
        float temp = 0.0f;
        if (std::scanf("%d %f %d %d", &n, &temp, &top_k, &rule) != 4 || n <= 0) return 1;
        std::vector<float> logits(n);
        for (int i = 0; i < n; ++i)
            if (std::scanf("%a", &logits[i]) != 1) return 1;
        int tok;
        if (rule) {
            const int top1 = static_cast<int>(std::max_element(logits.begin(), logits.end()) - logits.begin());
            tok = (top1 == 3 || top1 == 0) ? top1 : draw(logits, temp, top_k, rng);
        } else {
            tok = draw(logits, temp, top_k, rng);
        }
        std::printf("%d\n", tok);
    }
    return 0;
}
