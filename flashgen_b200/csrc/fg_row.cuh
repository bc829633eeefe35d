// fg_row.cuh — per-row semantics shared by the batch kernel (fg_stream.cuh)
// and the cluster kernel (fg_cluster.cuh): parameters, penalties, the exact
// temperature division, integer masses, and row geometry.
//
// Reference semantics (FlashGen):
//   flashgen/sampling/sampler.py:57-169   Sampler.sample / _sample_one /
//                                          _top_k_filter / _top_p_filter /
//                                          apply_repetition_penalty
//   csrc/runtime/pipeline.cpp:267-342      InferenceEngine::sample_tokens
#pragma once

#include "fg_common.cuh"

namespace fg {

constexpr float kL2E = 1.4426950408889634f;

__device__ __forceinline__ float ex2f_approx(float v) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(v));
    return y;
}

// out_ids value the batch kernel leaves on a row it hands to the cluster
// kernel (never a valid id, never the error id -1).
constexpr int64_t kDeferredId = -2;

// Row classes.
enum RowClass : int {
    RC_GREEDY = 0,   // greedy or temperature 0: first argmax of the penalised logits
    RC_TOPK = 1,     // top_k > 0 (then top-p on the k-filtered set)
    RC_NUCLEUS = 2,  // top_k off, 0 < top_p < 1
    RC_FULL = 3,     // top_k off, top_p == 1: draw over the whole row
};

// Per-row parameters, identical in every thread of a CTA.
struct RowP {
    int cls;
    int K;            // top-k (RC_TOPK): min(top_k, vocab)
    bool use_p;       // 0 < top_p < 1
    bool pen, rep_on, pres_on, freq_on;
    bool temp_on;     // y = x / T (T != 1)
    float T, rT, top_p, rep, pres, freq, u;
    int bad;          // FG_ROW_BAD_PARAM | FG_ROW_BAD_UNIFORM
};

// The parameters of caller row q. `hist_rows`: whether the row has a
// non-empty history and penalties are configured for the call.
__device__ __forceinline__ RowP load_row_params(const float* temperature, const float* top_p, const int32_t* top_k,
                                                const float* rep, const float* pres, const float* freq,
                                                const uint8_t* greedy, const float* uniforms, int q,
                                                bool has_hist, int vocab) {
    RowP p;
    p.T = __ldg(temperature + q);
    p.top_p = __ldg(top_p + q);
    const int tk = __ldg(top_k + q);
    p.rep = rep ? __ldg(rep + q) : 1.0f;
    p.pres = pres ? __ldg(pres + q) : 0.0f;
    p.freq = freq ? __ldg(freq + q) : 0.0f;
    const bool g = greedy ? (__ldg(greedy + q) != 0) : false;
    p.u = __ldg(uniforms + q);
    p.bad = 0;
    p.rep_on = has_hist && (p.rep != 1.0f);
    p.freq_on = has_hist && (p.freq != 0.0f);
    p.pres_on = has_hist && (p.pres != 0.0f);
    p.pen = p.rep_on || p.freq_on || p.pres_on;
    if (!(p.rep == p.rep) || !(p.pres == p.pres) || !(p.freq == p.freq)) p.bad |= FG_ROW_BAD_PARAM;
    p.K = 1;
    p.use_p = false;
    p.temp_on = false;
    p.rT = 1.0f;
    if (g || p.T == 0.0f) {
        p.cls = RC_GREEDY;
        return p;
    }
    if (!(p.T > 0.0f) || !(p.top_p > 0.0f && p.top_p <= 1.0f)) p.bad |= FG_ROW_BAD_PARAM;
    if (!(p.u >= 0.0f && p.u < 1.0f)) p.bad |= FG_ROW_BAD_UNIFORM;
    p.temp_on = (p.T != 1.0f);
    p.rT = p.temp_on ? __frcp_rn(p.T) : 1.0f;
    p.use_p = (p.top_p > 0.0f && p.top_p < 1.0f);
    if (tk > 0) {
        p.cls = RC_TOPK;
        p.K = tk < vocab ? tk : vocab;
    } else {
        p.cls = p.use_p ? RC_NUCLEUS : RC_FULL;
        p.K = vocab;
    }
    return p;
}

// y = x / T, bit-identical to IEEE fp32 division (sampler.py:108-109).
__device__ __forceinline__ float ydiv(const RowP& p, float x) { return p.temp_on ? div_rn(x, p.T, p.rT) : x; }

// Penalised value of a history column with `count` occurrences:
// repetition (sampler.py:134-146, on unique ids), then frequency and
// presence, each an fp32 operation in that order.
__device__ __forceinline__ float penalize(const RowP& p, float x, uint32_t count) {
    if (p.rep_on) x = (x > 0.0f) ? __fdiv_rn(x, p.rep) : __fmul_rn(x, p.rep);
    if (p.freq_on) x = __fsub_rn(x, __fmul_rn(p.freq, (float)count));
    if (p.pres_on) x = __fsub_rn(x, p.pres);
    return x;
}

// Integer mass of a token with scaled value y: round(2^S * e^(y - My)). Equal
// y give equal masses, so ties share one mass and sums are exact.
__device__ __forceinline__ uint64_t qmass(float y, float My, float scale) {
    return (uint64_t)__float2ull_rn(expf(y - My) * scale);
}

// Smallest float x' <= tau with y(x') >= y(tau): the filter bound in x that
// keeps every element tying with tau after the division by T.
__device__ __forceinline__ float xmin_for_y(const RowP& p, float tau) {
    if (!p.temp_on || !(tau > -INFINITY) || !(tau < INFINITY)) return tau;
    const float yt = ydiv(p, tau);
    uint32_t k = fkey(tau);
    for (int steps = 0; steps < 8; ++steps) {
        if (k <= KEY_NEG_INF) return funkey(k);
        if (ydiv(p, funkey(k - 1)) >= yt) --k; else return funkey(k);
    }
    uint32_t lo = KEY_NEG_INF, hi = k;
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo) / 2;
        if (ydiv(p, funkey(mid)) >= yt) hi = mid; else lo = mid + 1;
    }
    return funkey(hi);
}

// Row geometry: the 16-byte-aligned interior (bulk-copied), and the ragged
// columns before and after it (< 16 bytes each, loaded one by one).
struct Geom {
    const uint8_t* row;        // column 0
    const uint8_t* interior;   // first aligned byte
    int64_t ibytes;            // interior bytes (multiple of 16)
    int head;                  // columns before the interior
    int tail0;                 // first column after the interior
};
template <int ESZ>
__device__ __forceinline__ Geom row_geom(const void* logits, int64_t row_stride, int vocab, int r) {
    Geom g;
    g.row = reinterpret_cast<const uint8_t*>(logits) + (int64_t)r * row_stride * ESZ;
    const uint8_t* end = g.row + (int64_t)vocab * ESZ;
    const uintptr_t a0 = (reinterpret_cast<uintptr_t>(g.row) + 15) & ~uintptr_t(15);
    const uintptr_t a1 = reinterpret_cast<uintptr_t>(end) & ~uintptr_t(15);
    if (a1 <= a0) {
        g.interior = g.row; g.ibytes = 0; g.head = vocab; g.tail0 = vocab;
        return g;
    }
    g.interior = reinterpret_cast<const uint8_t*>(a0);
    g.ibytes = (int64_t)(a1 - a0);
    g.head = (int)((a0 - reinterpret_cast<uintptr_t>(g.row)) / ESZ);
    g.tail0 = g.head + (int)(g.ibytes / ESZ);
    return g;
}

// Hash slot of a column in an open-addressed table of `mask + 1` slots (a
// power of two): the top bits of Knuth's multiplicative hash, which depend on
// every bit of the column.
__device__ __forceinline__ uint32_t col_hash(uint32_t c, uint32_t mask) {
    const uint32_t bits = 32u - __clz(mask);
    return bits == 0u ? 0u : ((c * 2654435761u) >> (32u - bits)) & mask;
}
constexpr uint32_t kEmptySlot = 0xffffffffu;

}  // namespace fg
