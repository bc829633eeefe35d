// fg_sample_kernel.cuh — fused decode-step sampler for sm_100a.
//
// One persistent CTA per SM walks rows r = blockIdx.x, +gridDim.x, ...
//   warp NCW (producer): streams each row's 16-byte-aligned interior from HBM
//     into a shared-memory ring of TILE_BYTES stages with 1-D bulk async copies
//     (cp.async.bulk, completion on mbarriers);
//   warps 0..NCW-1 (consumers): per row
//     1. history prologue: bitmap of history ids (+ word prefix and counts when
//        a frequency penalty is set), all in shared memory;
//     2. single pass over the row: penalties at history ids, NaN-propagating
//        max, online sum-exp (rows whose top-p runs over the whole
//        vocabulary), and a candidate filter x >= xmin that appends
//        (key, column) pairs to a shared buffer; xmin is a running lower bound
//        on the K-th largest value, raised by periodic compactions;
//     3. epilogue over the candidates: exact top-k threshold, fixed-point
//        masses, top-p cut (ties in ascending id order), inverse-CDF draw —
//        all as block radix selects over integer histograms, so the result does
//        not depend on thread scheduling;
//     4. general path when the candidates cannot decide the row (nucleus
//        deeper than the candidates, ties beyond capacity, top_k above the
//        on-chip limit, NaN rows, no filter at all): the same selects run over
//        the whole row re-read from global memory (L2-resident after step 2).
//
// Reference semantics (FlashGen): flashgen/sampling/sampler.py:57-169,
// csrc/runtime/pipeline.cpp:267-342.
#pragma once

#include "fg_common.cuh"

namespace fg {

constexpr int NCW = 16;                 // consumer warps
constexpr int NCT = NCW * 32;           // consumer threads
constexpr int NTHREADS = NCT + 32;      // + one producer warp
constexpr int TILE_ELEMS = 4096;        // elements per ring stage
constexpr int CHECK_TILES = 2;          // tiles between compaction checks
constexpr int CAND_CAP = 12288;         // candidate buffer entries
constexpr int HWM = CAND_CAP - CHECK_TILES * TILE_ELEMS - 64;  // compaction trigger
constexpr int K_FAST_MAX = 2048;        // largest top_k decided on the candidates
constexpr int K_NUCLEUS = 2048;         // candidate target for top-p-only rows
constexpr int Q_CAP = 4096;             // kept entries whose masses fit on chip
constexpr int BAR_CONS = 1;             // named barrier of the consumer warps
constexpr int NBINS = 256;

enum Mode : int { MODE_GREEDY = 0, MODE_TOPK = 1, MODE_NUCLEUS = 2, MODE_FULL = 3 };

struct KParams {
    const void* logits;
    int64_t row_stride;
    int32_t batch, vocab;
    int64_t vocab_offset, vocab_total;
    const int32_t* hist_ids;
    const int64_t* hist_offsets;
    const float* temperature;
    const float* top_p;
    const int32_t* top_k;
    const float* rep;
    const float* pres;
    const float* freq;
    const uint8_t* greedy;
    const float* uniforms;
    int64_t* out_ids;
    int32_t* out_status;
    float* out_probs;
    // shared-memory layout (byte offsets into dynamic smem)
    int32_t nstage;
    int32_t nwords;          // bitmap words
    int32_t hu_cap;          // count-table entries (0: no frequency penalty)
    int32_t off_bitmap, off_prefix, off_counts, off_ring;
    int32_t pen_possible;    // history + some penalty array present
    int32_t mass_shift;      // S: masses are round(e * 2^S)
    int32_t id_bits;         // bits needed for a column index
};

struct RowCtl {
    uint32_t n;          // candidates
    uint32_t hikey;      // max key appended
    float xmin;          // candidate filter (x >= xmin)
    int cand_on;
    int status;
    int general;         // row needs the general path
    int abort;           // pipeline gave up (timeout)
    // selection results / broadcast slots
    uint32_t sel_digit;
    int sel_ok;
    uint64_t sel_before, sel_at;
    uint32_t sel_nat;
    uint32_t u32a, u32b;
    float f32a;
    double f64a;
};

struct Smem {
    uint64_t* full;
    uint64_t* empty;
    RowCtl* ctl;
    uint64_t* red64;     // [NCW]
    float* redf;         // [NCW]
    uint32_t* red32;     // [NCW]
    double* redd;        // [NCW]
    unsigned long long* bins;  // [NBINS]
    uint32_t* cnts;      // [NBINS]
    uint32_t* ckey;      // [CAND_CAP]
    uint32_t* cid;       // [CAND_CAP]
    uint64_t* q;         // [Q_CAP] (aliases ckey[Q_CAP..])
    uint32_t* bitmap;
    uint32_t* prefix;
    uint32_t* counts;
    uint8_t* ring;
};

__host__ __device__ inline int align_up_i(int x, int a) { return (x + a - 1) / a * a; }

// Fixed part of the layout (everything except bars, penalty tables and ring).
struct FixedLayout {
    int ctl, red64, redf, red32, redd, bins, cnts, ckey, cid, end;
};
__host__ __device__ inline FixedLayout fixed_layout(int nstage) {
    FixedLayout L;
    int o = 16 * nstage;  // full[nstage] + empty[nstage]
    o = align_up_i(o, 16); L.ctl = o; o += (int)sizeof(RowCtl);
    o = align_up_i(o, 16); L.red64 = o; o += 8 * NCW;
    L.redf = o; o += 4 * NCW;
    L.red32 = o; o += 4 * NCW;
    o = align_up_i(o, 8); L.redd = o; o += 8 * NCW;
    o = align_up_i(o, 16); L.bins = o; o += 8 * NBINS;
    L.cnts = o; o += 4 * NBINS;
    o = align_up_i(o, 16); L.ckey = o; o += 4 * CAND_CAP;
    L.cid = o; o += 4 * CAND_CAP;
    L.end = o;
    return L;
}

__device__ __forceinline__ Smem carve(uint8_t* base, const KParams& P) {
    FixedLayout L = fixed_layout(P.nstage);
    Smem s;
    s.full = reinterpret_cast<uint64_t*>(base);
    s.empty = s.full + P.nstage;
    s.ctl = reinterpret_cast<RowCtl*>(base + L.ctl);
    s.red64 = reinterpret_cast<uint64_t*>(base + L.red64);
    s.redf = reinterpret_cast<float*>(base + L.redf);
    s.red32 = reinterpret_cast<uint32_t*>(base + L.red32);
    s.redd = reinterpret_cast<double*>(base + L.redd);
    s.bins = reinterpret_cast<unsigned long long*>(base + L.bins);
    s.cnts = reinterpret_cast<uint32_t*>(base + L.cnts);
    s.ckey = reinterpret_cast<uint32_t*>(base + L.ckey);
    s.cid = reinterpret_cast<uint32_t*>(base + L.cid);
    s.q = reinterpret_cast<uint64_t*>(base + L.ckey + 4 * Q_CAP);
    s.bitmap = reinterpret_cast<uint32_t*>(base + P.off_bitmap);
    s.prefix = reinterpret_cast<uint32_t*>(base + P.off_prefix);
    s.counts = reinterpret_cast<uint32_t*>(base + P.off_counts);
    s.ring = base + P.off_ring;
    return s;
}

// Row geometry: 16-byte-aligned interior streamed by the producer, ragged
// head/tail columns loaded directly by the consumers.
struct RowGeom {
    const uint8_t* interior;   // first aligned byte
    int64_t interior_bytes;    // multiple of 16
    int head;                  // columns before the interior
    int tail0;                 // first column after the interior
    int ntiles;
};
template <int ESZ>
__device__ __forceinline__ RowGeom row_geom(const KParams& P, int r) {
    RowGeom g;
    const uint8_t* start = reinterpret_cast<const uint8_t*>(P.logits) + (int64_t)r * P.row_stride * ESZ;
    const uint8_t* end = start + (int64_t)P.vocab * ESZ;
    uintptr_t a0 = (reinterpret_cast<uintptr_t>(start) + 15) & ~uintptr_t(15);
    uintptr_t a1 = reinterpret_cast<uintptr_t>(end) & ~uintptr_t(15);
    if (a1 <= a0) {
        g.interior = start; g.interior_bytes = 0; g.head = P.vocab; g.tail0 = P.vocab; g.ntiles = 0;
        return g;
    }
    g.interior = reinterpret_cast<const uint8_t*>(a0);
    g.interior_bytes = (int64_t)(a1 - a0);
    g.head = (int)((a0 - reinterpret_cast<uintptr_t>(start)) / ESZ);
    g.tail0 = g.head + (int)(g.interior_bytes / ESZ);
    constexpr int64_t TB = (int64_t)TILE_ELEMS * ESZ;
    g.ntiles = (int)((g.interior_bytes + TB - 1) / TB);
    return g;
}

// ---------------------------------------------------------------------------
// Per-row parameters (registers, identical in every consumer thread)
// ---------------------------------------------------------------------------
struct RowParams {
    int mode;
    int K;           // top-k (TOPK), candidate target otherwise
    bool use_p;
    bool cand;       // candidate filter requested
    bool pen, freq_on, pres_on, rep_on;
    bool temp_on;    // y = x / T
    float T, rT, top_p, rep, pres, freq, u;
    float c;         // log2(e) / T for the online sum-exp
    int bad;         // FG_ROW_BAD_PARAM / FG_ROW_BAD_UNIFORM
};

__device__ __forceinline__ RowParams row_params(const KParams& P, int r) {
    RowParams p;
    p.T = __ldg(P.temperature + r);
    p.top_p = __ldg(P.top_p + r);
    int tk = __ldg(P.top_k + r);
    p.rep = P.rep ? __ldg(P.rep + r) : 1.0f;
    p.pres = P.pres ? __ldg(P.pres + r) : 0.0f;
    p.freq = P.freq ? __ldg(P.freq + r) : 0.0f;
    bool g = P.greedy ? (__ldg(P.greedy + r) != 0) : false;
    p.u = __ldg(P.uniforms + r);
    p.bad = 0;
    bool hist = P.pen_possible && P.hist_offsets != nullptr &&
                (__ldg(P.hist_offsets + r + 1) > __ldg(P.hist_offsets + r));
    p.rep_on = hist && (p.rep != 1.0f);
    p.freq_on = hist && (p.freq != 0.0f) && P.hu_cap > 0;
    p.pres_on = hist && (p.pres != 0.0f);
    p.pen = p.rep_on || p.freq_on || p.pres_on;
    if (!(p.rep == p.rep) || !(p.pres == p.pres) || !(p.freq == p.freq)) p.bad |= FG_ROW_BAD_PARAM;
    if (g || p.T == 0.0f) {
        p.mode = MODE_GREEDY; p.K = 1; p.use_p = false; p.cand = true; p.temp_on = false;
        p.rT = 1.0f; p.c = 1.4426950408889634f;
        return p;
    }
    if (!(p.T > 0.0f) || !(p.top_p > 0.0f && p.top_p <= 1.0f)) p.bad |= FG_ROW_BAD_PARAM;
    if (!(p.u >= 0.0f && p.u < 1.0f)) p.bad |= FG_ROW_BAD_UNIFORM;
    p.temp_on = (p.T != 1.0f);
    p.rT = p.temp_on ? __frcp_rn(p.T) : 1.0f;
    p.c = p.temp_on ? __fdiv_rn(1.4426950408889634f, p.T) : 1.4426950408889634f;
    p.use_p = (p.top_p > 0.0f && p.top_p < 1.0f);
    if (tk > 0) {
        p.mode = MODE_TOPK;
        p.K = tk < P.vocab ? tk : P.vocab;
        p.cand = (p.K <= K_FAST_MAX);
    } else if (p.use_p) {
        p.mode = MODE_NUCLEUS; p.K = K_NUCLEUS; p.cand = true;
    } else {
        p.mode = MODE_FULL; p.K = 0; p.cand = false;
    }
    return p;
}

__device__ __forceinline__ float ydiv(const RowParams& p, float x) {
    return p.temp_on ? div_rn(x, p.T, p.rT) : x;
}

// Smallest float x' <= tau such that y(x') >= y(tau): the candidate filter in
// x-space that keeps every element whose temperature-scaled value ties with or
// exceeds that of tau.
__device__ float xmin_for(const RowParams& p, float tau) {
    if (!p.temp_on || !(tau > -INFINITY)) return tau;
    const float yt = ydiv(p, tau);
    uint32_t k = fkey(tau);
    int steps = 0;
    while (k > KEY_NEG_INF && steps < 8) {
        float xp = funkey(k - 1);
        if (ydiv(p, xp) >= yt) { --k; ++steps; } else return funkey(k);
    }
    if (k <= KEY_NEG_INF) return funkey(k);
    // long run of x values with the same quotient: binary search below k
    uint32_t lo = KEY_NEG_INF, hi = k;   // pred(hi) true; find smallest true
    while (lo < hi) {
        uint32_t mid = lo + (hi - lo) / 2;
        if (ydiv(p, funkey(mid)) >= yt) hi = mid; else lo = mid + 1;
    }
    return funkey(hi);
}

// ---------------------------------------------------------------------------
// Consumer-group reductions (named barrier BAR_CONS, NCT threads)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void csync() { named_sync(BAR_CONS, NCT); }

__device__ __forceinline__ float cons_max_nan(float v, const Smem& s, int tid) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((tid & 31) == 0) s.redf[tid >> 5] = v;
    csync();
    float r = s.redf[0];
#pragma unroll
    for (int w = 1; w < NCW; ++w) r = fmax_nan(r, s.redf[w]);
    csync();
    return r;
}
__device__ __forceinline__ uint64_t cons_sum_u64(uint64_t v, const Smem& s, int tid) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += shfl_u64(v, (tid & 31) ^ o);
    if ((tid & 31) == 0) s.red64[tid >> 5] = v;
    csync();
    uint64_t r = 0;
#pragma unroll
    for (int w = 0; w < NCW; ++w) r += s.red64[w];
    csync();
    return r;
}
__device__ __forceinline__ uint32_t cons_min_u32(uint32_t v, const Smem& s, int tid) {
    v = __reduce_min_sync(0xffffffffu, v);
    if ((tid & 31) == 0) s.red32[tid >> 5] = v;
    csync();
    uint32_t r = s.red32[0];
#pragma unroll
    for (int w = 1; w < NCW; ++w) r = min(r, s.red32[w]);
    csync();
    return r;
}
__device__ __forceinline__ uint32_t cons_max_u32(uint32_t v, const Smem& s, int tid) {
    v = __reduce_max_sync(0xffffffffu, v);
    if ((tid & 31) == 0) s.red32[tid >> 5] = v;
    csync();
    uint32_t r = s.red32[0];
#pragma unroll
    for (int w = 1; w < NCW; ++w) r = max(r, s.red32[w]);
    csync();
    return r;
}
// Deterministic double sum: fixed shuffle tree, then warps in index order.
__device__ __forceinline__ double cons_sum_f64(double v, const Smem& s, int tid) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((tid & 31) == 0) s.redd[tid >> 5] = v;
    csync();
    double r = 0.0;
#pragma unroll
    for (int w = 0; w < NCW; ++w) r += s.redd[w];
    csync();
    return r;
}
// Exclusive prefix over consumer threads (thread order), returns (excl, total).
__device__ __forceinline__ uint32_t cons_excl_scan_u32(uint32_t v, uint32_t& total, const Smem& s, int tid) {
    const int lane = tid & 31, w = tid >> 5;
    uint32_t incl = warp_incl_scan_u32(v, lane);
    if (lane == 31) s.red32[w] = incl;
    csync();
    uint32_t base = 0, tot = 0;
#pragma unroll
    for (int i = 0; i < NCW; ++i) {
        uint32_t t = s.red32[i];
        if (i < w) base += t;
        tot += t;
    }
    csync();
    total = tot;
    return base + incl - v;
}

// ---------------------------------------------------------------------------
// Block radix select.
//
// Over the multiset of (key, weight) pairs that `enumerate` yields in this
// thread (every consumer thread yields its own share), find the key k* such
// that  W(before k*) <= target < W(before k*) + W(at k*), where "before" means
// larger keys (DESC) or smaller keys (ASC). Weights are summed exactly in
// integers, so the answer does not depend on thread scheduling. COUNT selects
// use weight 1 (the caller's weight argument is ignored).
// Returns ok=false when target >= total weight.
// ---------------------------------------------------------------------------
struct SelOut {
    uint32_t key;
    uint64_t before;   // weight strictly before key*
    uint64_t at;       // weight at key*
    uint32_t n_at;     // elements at key*
    bool ok;
};

template <bool DESC, bool COUNT, class Enum>
__device__ SelOut block_select(Enum&& enumerate, uint64_t target, int key_bits, const Smem& s, int tid) {
    SelOut out;
    uint32_t prefix = 0, pmask = 0;
    uint64_t before = 0;
    int rem = key_bits;
    bool ok = true;
    uint64_t at = 0; uint32_t nat = 0;
    while (rem > 0) {
        const int w = rem < 8 ? rem : 8;
        const int shift = rem - w;
        const uint32_t dmask = (1u << w) - 1u;
        if (tid < NBINS) { s.cnts[tid] = 0; if (!COUNT) s.bins[tid] = 0ull; }
        csync();
        enumerate([&](uint32_t k, uint64_t wt) {
            if ((k & pmask) == prefix) {
                uint32_t d = (k >> shift) & dmask;
                atomicAdd(&s.cnts[d], 1u);
                if (!COUNT) atomicAdd(&s.bins[d], (unsigned long long)wt);
            }
        });
        csync();
        if (tid < 32) {
            const int lane = tid;
            // lane covers 8 consecutive bins in scan order
            uint64_t v[8];
            uint64_t lsum = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                int o = lane * 8 + j;
                int d = DESC ? (NBINS - 1 - o) : o;
                uint64_t x = COUNT ? (uint64_t)s.cnts[d] : (uint64_t)s.bins[d];
                v[j] = x; lsum += x;
            }
            uint64_t incl = warp_incl_scan_u64(lsum, lane);
            uint64_t excl = incl - lsum;
            uint64_t rel = target - before;  // target >= before by construction
            bool mine = (excl <= rel) && (rel < incl);
            uint32_t bal = __ballot_sync(0xffffffffu, mine);
            if (bal == 0) {
                if (lane == 0) { s.ctl->sel_ok = 0; s.ctl->sel_digit = 0; s.ctl->sel_before = 0; }
            } else if (lane == __ffs(bal) - 1) {
                uint64_t c = excl;
                int jj = 0;
                for (; jj < 7; ++jj) {
                    if (rel < c + v[jj]) break;
                    c += v[jj];
                }
                int o = lane * 8 + jj;
                int d = DESC ? (NBINS - 1 - o) : o;
                s.ctl->sel_ok = 1;
                s.ctl->sel_digit = (uint32_t)d;
                s.ctl->sel_before = c;
            }
        }
        csync();
        if (!s.ctl->sel_ok) { ok = false; }
        const uint32_t d = s.ctl->sel_digit;
        before += s.ctl->sel_before;
        nat = s.cnts[d];
        at = COUNT ? (uint64_t)nat : (uint64_t)s.bins[d];
        csync();
        if (!ok) break;
        prefix |= d << shift;
        pmask |= dmask << shift;
        rem = shift;
    }
    out.key = prefix; out.before = before; out.at = at; out.n_at = nat; out.ok = ok;
    return out;
}

}  // namespace fg
