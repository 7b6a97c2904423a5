// The library's stochastic decoding rule (include/speculative.h) on the
// host, for logits that a caller's own target / base function returns:
// integer nucleus weights with exact sums and Philox-keyed inverse-CDF
// draws, the same operations as the device sampler (sample_ops.cu), so a
// host draw and a device draw from the same logits are the same token.
#pragma once

#include <math.h>
#include <stdint.h>

#include <vector>

#include "fl_cuda.h"

namespace fl_host {

// E = trunc(e^x * 2^24) for x = (l - max) / T <= 0, 0 below x = -17: e^x by
// Cody-Waite reduction x = k ln2 + r (ln2 as a 16-bit head plus a float
// tail) and the degree-7 Taylor polynomial of e^r in Horner form, each step
// one correctly rounded fma or multiply, then the exact scale 2^(k + 24).
inline uint32_t weight(float x) {
    if (!(x >= -17.0f)) return 0u;
    const float kf = rintf(x * 1.442695f);
    float r = fmaf(-kf, 0.693145751953125f, x);
    r = fmaf(-kf, 1.4286068e-06f, r);
    float p = 0.0001984127f;
    p = fmaf(p, r, 0.0013888889f);
    p = fmaf(p, r, 0.008333334f);
    p = fmaf(p, r, 0.041666668f);
    p = fmaf(p, r, 0.16666667f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const uint32_t E = (uint32_t)ldexpf(p, (int)kf + 24);
    return E > (1u << 24) ? (1u << 24) : E;
}

// Nucleus weights of logits l: E_i = weight((l_i - max) / T); kept are the
// E_i >= t*, t* the largest integer whose kept mass reaches
// max(1, trunc(top_p * 2^24)) / 2^24 of the total. Returns the kept mass.
inline uint64_t weights(const float* l, int V, float T, float top_p, std::vector<uint32_t>& E) {
    E.resize(V);
    float mx = l[0];
    for (int i = 1; i < V; i++) mx = l[i] > mx ? l[i] : mx;
    uint64_t z = 0;
    for (int i = 0; i < V; i++) {
        E[i] = weight((l[i] - mx) / T);
        z += E[i];
    }
    uint32_t P = (uint32_t)(top_p * 16777216.0f);
    if (P < 1u) P = 1u;
    const unsigned __int128 need = (unsigned __int128)P * z;
    uint32_t lo = 1u, hi = (1u << 24) + 1u;
    while (hi - lo > 1u) {
        const uint32_t mid = lo + (hi - lo) / 2u;
        uint64_t s = 0;
        for (int i = 0; i < V; i++)
            if (E[i] >= mid) s += E[i];
        if (((unsigned __int128)s << 24) >= need) lo = mid;
        else hi = mid;
    }
    uint64_t M = 0;
    for (int i = 0; i < V; i++) {
        if (E[i] < lo) E[i] = 0u;
        M += E[i];
    }
    return M;
}

// First index whose running weight sum exceeds trunc(U * total / 2^24).
inline int pick(const std::vector<uint32_t>& w, uint64_t total, uint32_t U, int skip = -1) {
    const uint64_t tgt = (uint64_t)(((unsigned __int128)U * total) >> 24);
    uint64_t c = 0;
    for (int i = 0; i < (int)w.size(); i++) {
        if (i == skip) continue;
        c += w[i];
        if (c > tgt) return i;
    }
    return (int)w.size() - 1;
}

// 24 bits of Philox4x32-10 keyed (seed, 0) at counter (seq, step, pos, purpose).
inline uint32_t u24(uint32_t seed, uint32_t seq, uint32_t step, uint32_t pos, uint32_t purpose) {
    const uint32_t ctr[4] = {seq, step, pos, purpose};
    const uint32_t key[2] = {seed, 0u};
    uint32_t o[4];
    fl_philox4x32_10(ctr, key, o);
    return o[0] >> 8;
}

inline int argmax(const float* l, int V) {
    int b = 0;
    for (int i = 1; i < V; i++)
        if (l[i] > l[b]) b = i;
    return b;
}

}  // namespace fl_host
