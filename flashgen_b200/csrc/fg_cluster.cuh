// fg_cluster.cuh — the general row sampler: one thread-block cluster per row.
//
// A cluster of G CTAs (G <= 16) samples one row at a time. CTA s owns a
// contiguous slice of the row's columns. The first pass reads the slice from
// HBM once, applies the penalties and the temperature, and keeps the order-
// preserving key of every scaled value y = x / T in shared memory (the key
// cache), so every later pass is integer work on on-chip memory.
//
// Every decision is a "window query" over the keys of the row, by count
// (top-k) or by exact integer mass (top-p cut, draw):
//   1. each CTA histograms its keys into NBL bins of a key range (the bin is
//      the key's offset in the range, shifted), with counts and 64-bit masses;
//   2. the bins are reduced over the cluster through distributed shared
//      memory: CTA q sums the bins it owns over every peer, then every CTA
//      reads all reduced bins and scans them identically;
//   3. if the bin that holds the target has at most WMAX elements, each CTA
//      collects its elements of that bin (key, column), every CTA gathers the
//      G lists, and the element is selected exactly in shared memory (radix
//      select on the key, then on the column among ties); otherwise the bin's
//      key range is histogrammed again, finer.
// Masses are round(e^(y - My) * 2^S) in integers, so every sum is exact and
// the result does not depend on scheduling or on G.
//
// Chain per row (flashgen/sampling/sampler.py:57-169; draw order of
// csrc/runtime/pipeline.cpp:311-340): history (slice-local counts and
// penalised values of the row's history ids) -> pass 1 (maximum, first
// argmax, first NaN, key cache) -> top-k (K-th largest by count) -> top-p
// cut and the draw predicted from it (one query, two targets) -> the drawn
// column. The draw is queried again, exactly, only when the prediction
// missed its bin.
//
// This kernel samples small batches whole (a batch that would leave most SMs
// idle with one CTA per row) and the rows the batch kernel hands over
// (out_ids == kDeferredId): deep nuclei, large top-k, candidate overflow, NaN
// in a greedy row; and every row when kept-set probabilities are requested.
#pragma once

#include <cooperative_groups.h>

#include "fg_row.cuh"

namespace fg {
namespace clus {

namespace cg = cooperative_groups;

constexpr int NT = 512;          // threads per CTA
constexpr int NW = NT / 32;
constexpr int NBL = 512;         // bins of a window-query level
constexpr int NB8 = 256;         // bins of a local radix step (8-bit digits)
constexpr int GMAX = 16;         // largest cluster
constexpr int WMAX = 2048;       // elements of a window gathered into every CTA
constexpr int CLAIM_CHUNK = 16;  // rows per claim when sampling deferred rows (<= 32)

struct Params {
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
    unsigned int* ws;          // [2] row claims, [3] finished clusters
    int32_t all_rows;          // 1: every row; 0: rows whose out_ids is kDeferredId
    int32_t pen_possible;
    int32_t hu_cap;            // bound on a row's distinct history ids
    int32_t hslots;            // hash slots (power of two >= 2 * hu_cap)
    int32_t mass_shift;        // S
    int32_t swords;            // slice bitmap words
    int32_t cache_words;       // key-cache capacity (columns of the largest slice)
    int32_t off_ctl, off_hist, off_full, off_own, off_wloc, off_wall, off_bitmap, off_hcol, off_hval, off_cache;
};

// Per-CTA values published to the peers (double-buffered by exchange parity).
struct Part {
    float mx;                  // NaN-propagating maximum
    float bv;                  // argmax value
    uint32_t bc;               // argmax column (first)
    uint32_t nan_col;          // first NaN column
    uint32_t flags;            // row status bits seen by this CTA
    uint32_t nloc[2];          // window elements collected, per target
    uint32_t pad;
};

struct SelRes {
    uint32_t key;
    uint32_t ok;
    uint32_t nat;
    uint32_t pad;
    unsigned long long before, at;
};

struct Ctl {
    int row;                   // claimed row (rank 0 publishes it)
    uint32_t pend_base, pend_mask, npend;
    Part part[2];
    SelRes sel;                // result of a local select step
    SelRes bsel[2];            // result of a bin scan, per target
    uint32_t red32[NW];
    float redf[NW];
    unsigned long long red64[NW];
    uint32_t ncoll;            // collection counter
    uint32_t nuniq;            // distinct history columns of the slice
    uint32_t wn[2];            // gathered window sizes, per target
    uint32_t wcnt[2];          // local collection counters, per target
    uint32_t tiecol[2];        // column of a tie found in this CTA, per target
};

extern __shared__ __align__(128) uint8_t csmem[];

struct Sm {
    Ctl* ctl;
    uint32_t* hist;            // [2 parity][2 targets][3: count, mass lo, mass hi][NBL] local bins
    uint32_t* own;             // [2 parity][2 targets][3][NBL / G] bins reduced by this CTA (max NBL)
    uint32_t* full;            // [2 targets][3][NBL] all reduced bins (local copy)
    uint32_t* wloc;            // [2 targets][2: key, col][WMAX] this CTA's window elements
    uint32_t* wall;            // [2 targets][2][WMAX] the gathered window
    uint32_t* bitmap;
    uint32_t* hcol;
    float* hval;
    uint32_t* cache;           // key cache (the history hash during the prologue)
};
__device__ __forceinline__ Sm carve(const Params& P) {
    Sm s;
    s.ctl = reinterpret_cast<Ctl*>(csmem + P.off_ctl);
    s.hist = reinterpret_cast<uint32_t*>(csmem + P.off_hist);
    s.own = reinterpret_cast<uint32_t*>(csmem + P.off_own);
    s.full = reinterpret_cast<uint32_t*>(csmem + P.off_full);
    s.wloc = reinterpret_cast<uint32_t*>(csmem + P.off_wloc);
    s.wall = reinterpret_cast<uint32_t*>(csmem + P.off_wall);
    s.bitmap = reinterpret_cast<uint32_t*>(csmem + P.off_bitmap);
    s.hcol = reinterpret_cast<uint32_t*>(csmem + P.off_hcol);
    s.hval = reinterpret_cast<float*>(csmem + P.off_hval);
    s.cache = reinterpret_cast<uint32_t*>(csmem + P.off_cache);
    return s;
}
__host__ __device__ inline int hist_words() { return 2 * 2 * 3 * NBL; }
__host__ __device__ inline int own_words(int G) { return 2 * 2 * 3 * (NBL / G); }
__host__ __device__ inline int full_words() { return 2 * 3 * NBL; }
__host__ __device__ inline int win_words() { return 2 * 2 * WMAX; }
__device__ __forceinline__ uint32_t* hist_ptr(const Sm& s, int par, int t, int a) {
    return s.hist + ((par * 2 + t) * 3 + a) * NBL;
}
// this CTA's reduced bins: per (parity, target, array) NBL / G words
__device__ __forceinline__ uint32_t* own_ptr(const Sm& s, int par, int t, int a, int per) {
    return s.own + ((par * 2 + t) * 3 + a) * per;
}
__device__ __forceinline__ uint32_t* full_ptr(const Sm& s, int t, int a) { return s.full + (t * 3 + a) * NBL; }
__device__ __forceinline__ uint32_t* wloc_ptr(const Sm& s, int t, int a) { return s.wloc + (t * 2 + a) * WMAX; }
__device__ __forceinline__ uint32_t* wall_ptr(const Sm& s, int t, int a) { return s.wall + (t * 2 + a) * WMAX; }

// ---------------------------------------------------------------------------
// Block reductions (all NT threads)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, const Sm& s) {
    v = __reduce_add_sync(0xffffffffu, v);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s.ctl->red32[w] = v;
    __syncthreads();
    uint32_t r = 0;
#pragma unroll
    for (int i = 0; i < NW; ++i) r += s.ctl->red32[i];
    __syncthreads();
    return r;
}
__device__ __forceinline__ uint32_t block_min_u32(uint32_t v, const Sm& s) {
    v = __reduce_min_sync(0xffffffffu, v);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s.ctl->red32[w] = v;
    __syncthreads();
    uint32_t r = 0xffffffffu;
#pragma unroll
    for (int i = 0; i < NW; ++i) r = min(r, s.ctl->red32[i]);
    __syncthreads();
    return r;
}
__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, const Sm& s) {
    v = __reduce_max_sync(0xffffffffu, v);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s.ctl->red32[w] = v;
    __syncthreads();
    uint32_t r = 0u;
#pragma unroll
    for (int i = 0; i < NW; ++i) r = max(r, s.ctl->red32[i]);
    __syncthreads();
    return r;
}
__device__ __forceinline__ float block_max_nan(float v, const Sm& s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s.ctl->redf[w] = v;
    __syncthreads();
    float r = s.ctl->redf[0];
#pragma unroll
    for (int i = 1; i < NW; ++i) r = fmax_nan(r, s.ctl->redf[i]);
    __syncthreads();
    return r;
}
// (v, c) beats (v2, c2) when v > v2, or v == v2 and c < c2: the first maximum
__device__ __forceinline__ bool arg_better(float v, uint32_t c, float v2, uint32_t c2) {
    return v > v2 || (v == v2 && c < c2);
}
__device__ __forceinline__ void block_argmax(float& v, uint32_t& c, const Sm& s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t c2 = __shfl_xor_sync(0xffffffffu, c, o);
        if (arg_better(v2, c2, v, c)) { v = v2; c = c2; }
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { s.ctl->redf[w] = v; s.ctl->red32[w] = c; }
    __syncthreads();
    float bv = s.ctl->redf[0];
    uint32_t bc = s.ctl->red32[0];
#pragma unroll
    for (int i = 1; i < NW; ++i)
        if (arg_better(s.ctl->redf[i], s.ctl->red32[i], bv, bc)) { bv = s.ctl->redf[i]; bc = s.ctl->red32[i]; }
    __syncthreads();
    v = bv;
    c = bc;
}
__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v, const Sm& s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += shfl_u64(v, (threadIdx.x & 31) ^ o);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s.ctl->red64[w] = v;
    __syncthreads();
    unsigned long long r = 0;
#pragma unroll
    for (int i = 0; i < NW; ++i) r += s.ctl->red64[i];
    __syncthreads();
    return r;
}

// 64-bit weight added to a bin as two 32-bit words with an exact carry
// (64-bit shared atomics serialise far more under contention).
__device__ __forceinline__ void add_w(uint32_t* lo, uint32_t* hi, uint32_t d, uint64_t w) {
    const uint32_t l = (uint32_t)w;
    uint32_t h = (uint32_t)(w >> 32);
    if (l) {
        const uint32_t old = atomicAdd(&lo[d], l);
        h += (old + l < old) ? 1u : 0u;
    }
    if (h) atomicAdd(&hi[d], h);
}

// Number of low bits that vary among keys in [lo, hi].
__device__ __forceinline__ int varying_bits(uint32_t lo, uint32_t hi) {
    const uint32_t d = lo ^ hi;
    return d == 0 ? 0 : 32 - __clz(d);
}

// ---------------------------------------------------------------------------
// Row slice of this CTA: interior chunks [ch0, ch1) plus, for the first and
// last rank, the ragged head and tail columns; columns [c_lo, c_hi).
// ---------------------------------------------------------------------------
struct Slice {
    int ch0, ch1;
    int c_lo, c_hi;
    bool head, tail;
};
template <int ESZ>
__device__ __forceinline__ Slice make_slice(const Geom& g, int vocab, int rank, int G) {
    constexpr int VEC = 16 / ESZ;
    const int nch = (int)(g.ibytes / 16);
    Slice sl;
    sl.ch0 = (int)((int64_t)nch * rank / G);
    sl.ch1 = (int)((int64_t)nch * (rank + 1) / G);
    sl.head = rank == 0;
    sl.tail = rank == G - 1;
    sl.c_lo = sl.head ? 0 : g.head + sl.ch0 * VEC;
    sl.c_hi = sl.tail ? vocab : g.head + sl.ch1 * VEC;
    return sl;
}

// ---------------------------------------------------------------------------
// History of the slice: distinct history columns in [c_lo, c_hi) with their
// counts (open-addressed hash laid over the key cache), their penalised
// values and a bitmap. Returns the number kept in the table; ORs
// FG_ROW_BAD_HISTORY / FG_ROW_BAD_PARAM into *flags.
// ---------------------------------------------------------------------------
template <int DT>
__device__ uint32_t slice_history(const Params& P, const Sm& s, const Geom& g, const Slice& sl, const RowP& p, int q,
                                  uint32_t* flags) {
    using E = Elem<DT>;
    const int tid = threadIdx.x;
    const uint32_t mask = (uint32_t)P.hslots - 1u;
    uint32_t* hkey = s.cache;
    uint32_t* hcnt = s.cache + P.hslots;
    for (int i = tid; i < P.hslots; i += NT) { hkey[i] = kEmptySlot; hcnt[i] = 0u; }
    if (tid == 0) s.ctl->ncoll = 0u;
    __syncthreads();
    const int64_t h0 = __ldg(P.hist_offsets + q), h1 = __ldg(P.hist_offsets + q + 1);
    uint32_t bad = 0;
    for (int64_t i = h0 + tid; i < h1; i += NT) {
        const int64_t gid = __ldg(P.hist_ids + i);
        if (gid < 0 || gid >= P.vocab_total) { bad |= FG_ROW_BAD_HISTORY; continue; }
        const int64_t c = gid - P.vocab_offset;
        if (c < sl.c_lo || c >= sl.c_hi) continue;
        const uint32_t cc = (uint32_t)c;
        uint32_t h = col_hash(cc, mask);
        bool done = false;
        for (int probe = 0; probe <= (int)mask; ++probe) {
            const uint32_t k = atomicCAS(&hkey[h], kEmptySlot, cc);
            if (k == kEmptySlot || k == cc) { atomicAdd(&hcnt[h], 1u); done = true; break; }
            h = (h + 1u) & mask;
        }
        if (!done) bad |= FG_ROW_BAD_PARAM;   // more distinct ids than hist_max_len allows
        const int o = (int)c - sl.c_lo;
        atomicOr(&s.bitmap[o >> 5], 1u << (o & 31));
    }
    if (bad) atomicOr(flags, bad);
    __syncthreads();
    for (int i = tid; i < P.hslots; i += NT) {
        const uint32_t c = hkey[i];
        if (c == kEmptySlot) continue;
        const uint32_t pos = atomicAdd(&s.ctl->ncoll, 1u);
        if (pos < (uint32_t)P.hu_cap) {
            s.hcol[pos] = c;
            s.hval[pos] = __uint_as_float(hcnt[i]);   // the count until penalised below
        } else {
            atomicOr(flags, (uint32_t)FG_ROW_BAD_PARAM);
        }
    }
    __syncthreads();
    const uint32_t nu = s.ctl->ncoll;
    if (tid == 0) s.ctl->nuniq = nu;
    const uint32_t U = min(nu, (uint32_t)P.hu_cap);
    for (uint32_t i = tid; i < U; i += NT) {
        const uint32_t c = s.hcol[i];
        s.hval[i] = penalize(p, E::load(g.row, c), __float_as_uint(s.hval[i]));
    }
    __syncthreads();
    return U;
}

// ---------------------------------------------------------------------------
// Window queries.
//
// A level histograms the keys of the slice in [klo, khi] (and passing `keep`)
// into NBL bins: bin = (key - klo) >> shift. Weight: 1, or the integer mass.
// ---------------------------------------------------------------------------
struct Level {
    uint32_t klo, khi;
    int shift;
};
__device__ __forceinline__ Level make_level(uint32_t klo, uint32_t khi) {
    Level L;
    L.klo = klo;
    L.khi = khi;
    const int vb = varying_bits(0u, khi - klo);
    int b = 0;
    while ((NBL >> b) > 1 && (1 << b) < NBL) ++b;   // log2(NBL)
    L.shift = vb > b ? vb - b : 0;
    return L;
}
__device__ __forceinline__ uint32_t bin_of(const Level& L, uint32_t k) { return (k - L.klo) >> L.shift; }
__device__ __forceinline__ uint32_t bin_lo_key(const Level& L, uint32_t b) { return L.klo + (b << L.shift); }
__device__ __forceinline__ uint32_t bin_hi_key(const Level& L, uint32_t b) {
    const uint64_t h = (uint64_t)L.klo + ((uint64_t)(b + 1) << L.shift) - 1ull;
    return (uint32_t)min(h, (uint64_t)L.khi);
}

// How a query's targets are set once the first level knows the filtered
// set's total weight Q.
enum TgtMode : int {
    TM_FIXED = 0,   // targets as given
    TM_CUT = 1,     // t0 = floor(top_p * Q) (the cut); t1 = floor(u * t0) (the draw, predicted)
    TM_DRAW = 2,    // t0 = min(floor(u * Q), Q - 1) (the draw without a cut)
};

// One target of a query.
struct Tgt {
    bool active;
    bool mass;
    uint64_t target;           // weight before the element sought (descending key order)
    Level L;
    // results
    bool ok;                   // the target lies inside the filtered set and its window was gathered
    uint64_t before;           // weight of keys above the window's bin
    uint64_t bin_at;           // weight in the bin
    uint32_t n;                // gathered window size
    bool gathered;             // the window of the target's bin is in wall
    // exact select (window_select)
    bool found;
    uint32_t key, col;
    uint64_t before_key, at_key;   // weight of keys > key, and at key
    uint32_t n_key;
};
__device__ __forceinline__ Tgt tgt(bool active, bool mass, uint64_t target) {
    Tgt t;
    t.active = active; t.mass = mass; t.target = target;
    t.ok = false; t.before = 0; t.bin_at = 0; t.n = 0; t.gathered = false; t.found = false;
    t.key = 0u; t.col = 0u; t.before_key = 0; t.at_key = 0; t.n_key = 0u;
    t.L.klo = 0u; t.L.khi = 0u; t.L.shift = 0;
    return t;
}

// Cluster reduction of one level's bins (local histograms of parity par):
// CTA q sums the bins it owns over every peer; then every CTA copies every
// reduced bin from its owner. Two cluster barriers.
__device__ __forceinline__ void reduce_level(cg::cluster_group& cl, const Sm& s, int par, int G, const Tgt (&t)[2]) {
    const int tid = threadIdx.x;
    const int rank = (int)cl.block_rank();
    const int per = NBL / G;
    cl.sync();
    for (int i = tid; i < 2 * per; i += NT) {
        const int tt = i / per, b = rank * per + (i % per);
        if (!t[tt].active) continue;
        uint32_t vc[GMAX], vl[GMAX], vh[GMAX];
#pragma unroll
        for (int r = 0; r < GMAX; ++r) {
            vc[r] = 0u; vl[r] = 0u; vh[r] = 0u;
            if (r < G) {
                const uint32_t* h = cl.map_shared_rank(hist_ptr(s, par, tt, 0), (unsigned)r);
                vc[r] = h[b];
                if (t[tt].mass) { vl[r] = h[NBL + b]; vh[r] = h[2 * NBL + b]; }
            }
        }
        uint32_t c = 0;
        unsigned long long m = 0;
#pragma unroll
        for (int r = 0; r < GMAX; ++r) { c += vc[r]; m += ((unsigned long long)vh[r] << 32) | vl[r]; }
        const int lb = b - rank * per;
        own_ptr(s, par, tt, 0, per)[lb] = c;
        own_ptr(s, par, tt, 1, per)[lb] = (uint32_t)m;
        own_ptr(s, par, tt, 2, per)[lb] = (uint32_t)(m >> 32);
    }
    cl.sync();
    for (int i = tid; i < 2 * NBL; i += NT) {
        const int tt = i / NBL, b = i % NBL;
        if (!t[tt].active) continue;
        const uint32_t* o = cl.map_shared_rank(own_ptr(s, par, tt, 0, per), (unsigned)(b / per));
        const int lb = b % per;
        full_ptr(s, tt, 0)[b] = o[lb];
        full_ptr(s, tt, 1)[b] = o[per + lb];
        full_ptr(s, tt, 2)[b] = o[2 * per + lb];
    }
    __syncthreads();
}

// Warp w < 2 scans target w's reduced bins in descending order for its
// target; the bin holding it goes to s.ctl->bsel[w].
__device__ __forceinline__ void scan_level(const Sm& s, const Tgt (&t)[2]) {
    const int tid = threadIdx.x;
    const int w = tid >> 5, lane = tid & 31;
    if (w < 2 && t[w].active) {
        const Tgt& T = t[w];
        constexpr int PL = NBL / 32;
        const uint32_t* f = full_ptr(s, w, 0);
        uint64_t v[PL];
        uint64_t lsum = 0;
#pragma unroll
        for (int j = 0; j < PL; ++j) {
            const int d = NBL - 1 - (lane * PL + j);
            v[j] = T.mass ? (((uint64_t)f[2 * NBL + d] << 32) | f[NBL + d]) : (uint64_t)f[d];
            lsum += v[j];
        }
        const uint64_t incl = warp_incl_scan_u64(lsum, lane);
        const uint64_t excl = incl - lsum;
        const uint64_t rel = T.target - T.before;
        const bool mine = excl <= rel && rel < incl;
        const uint32_t bal = __ballot_sync(0xffffffffu, mine);
        SelRes& o = s.ctl->bsel[w];
        if (bal == 0) {
            if (lane == 0) o.ok = 0u;
        } else if (lane == __ffs(bal) - 1) {
            uint64_t c = excl;
            int jj = 0;
#pragma unroll
            for (int j = 0; j < PL; ++j)
                if (jj == j && rel >= c + v[j]) { c += v[j]; jj = j + 1; }
            if (jj > PL - 1) jj = PL - 1;
            const int d = NBL - 1 - (lane * PL + jj);
            o.ok = 1u;
            o.key = (uint32_t)d;
            o.before = c;
            o.nat = f[d];
            o.at = T.mass ? (((uint64_t)f[2 * NBL + d] << 32) | f[NBL + d]) : (uint64_t)f[d];
        }
    }
    __syncthreads();
}

// The local radix select of the gathered window of target tt: the element
// at weight `rel` in descending key order, ties in ascending column order.
__device__ __forceinline__ void scan_local(const Sm& s, int nb, uint64_t rel, bool mass, bool asc) {
    // warp 0; bins in s.hist (scratch of parity-independent use: see caller)
    const int lane = threadIdx.x & 31;
    const uint32_t* cn = s.full;                 // count bins (scratch)
    const uint32_t* lo = s.full + NB8;
    const uint32_t* hi = s.full + 2 * NB8;
    uint64_t v[8];
    uint64_t lsum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int o = lane * 8 + j;
        const int d = asc ? o : nb - 1 - o;
        v[j] = (o < nb) ? (mass ? (((uint64_t)hi[d] << 32) | lo[d]) : (uint64_t)cn[d]) : 0ull;
        lsum += v[j];
    }
    const uint64_t incl = warp_incl_scan_u64(lsum, lane);
    const uint64_t excl = incl - lsum;
    const bool mine = excl <= rel && rel < incl;
    const uint32_t bal = __ballot_sync(0xffffffffu, mine);
    SelRes& o = s.ctl->sel;
    if (bal == 0) {
        if (lane == 0) o.ok = 0u;
    } else if (lane == __ffs(bal) - 1) {
        uint64_t c = excl;
        int jj = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (jj == j && rel >= c + v[j]) { c += v[j]; jj = j + 1; }
        if (jj > 7) jj = 7;
        const int d = asc ? lane * 8 + jj : nb - 1 - (lane * 8 + jj);
        o.ok = 1u;
        o.key = (uint32_t)d;
        o.before = c;
        o.nat = cn[d];
        o.at = mass ? (((uint64_t)hi[d] << 32) | lo[d]) : (uint64_t)cn[d];
    }
}

// Exact select in the gathered window (n entries of target tt): key by
// weight in descending order, then the column among that key's ties.
// Weight of an entry: 1, or qmass of its key.
__device__ void window_select(const Sm& s, int tt, uint64_t rel, float My, float scale, Tgt& T) {
    const uint32_t n = T.n;
    const bool mass = T.mass;
    const int tid = threadIdx.x;
    const uint32_t* wk = wall_ptr(s, tt, 0);
    const uint32_t* wc = wall_ptr(s, tt, 1);
    uint32_t* cn = s.full;
    uint32_t* lo = s.full + NB8;
    uint32_t* hi = s.full + 2 * NB8;
    // key range of the window
    uint32_t kmn = 0xffffffffu, kmx = 0u;
    for (uint32_t i = tid; i < n; i += NT) { kmn = min(kmn, wk[i]); kmx = max(kmx, wk[i]); }
    kmn = block_min_u32(kmn, s);
    kmx = block_max_u32(kmx, s);
    int rem = varying_bits(kmn, kmx);
    uint32_t pmask = rem >= 32 ? 0u : ~((1u << rem) - 1u);
    uint32_t prefix = kmn & pmask;
    uint64_t before = 0, at = 0;
    uint32_t nat = n;
    bool ok = n > 0;
    if (rem == 0) {
        // one key: its weight
        at = mass ? (uint64_t)n * qmass(funkey(kmn), My, scale) : (uint64_t)n;
        ok = ok && rel < at;
    }
    while (ok && rem > 0) {
        const int w = rem < 8 ? rem : 8;
        const int shift = rem - w;
        const uint32_t dmask = (1u << w) - 1u;
        for (int b = tid; b < NB8; b += NT) { cn[b] = 0u; lo[b] = 0u; hi[b] = 0u; }
        __syncthreads();
        for (uint32_t i = tid; i < n; i += NT) {
            const uint32_t k = wk[i];
            if ((k & pmask) != prefix) continue;
            const uint32_t d = (k >> shift) & dmask;
            atomicAdd(&cn[d], 1u);
            if (mass) add_w(lo, hi, d, qmass(funkey(k), My, scale));
        }
        __syncthreads();
        if (tid < 32) scan_local(s, 1 << w, rel - before, mass, false);
        __syncthreads();
        const SelRes r = s.ctl->sel;
        __syncthreads();
        if (!r.ok) { ok = false; break; }
        before += r.before;
        prefix |= r.key << shift;
        pmask |= dmask << shift;
        rem = shift;
        at = r.at;
        nat = r.nat;
    }
    T.found = false;
    if (!ok) return;
    const uint32_t key = prefix;
    const uint64_t q = nat ? at / nat : 0;
    uint64_t j = mass ? (q ? (rel - before) / q : 0) : (rel - before);
    if (j >= nat) j = nat ? nat - 1 : 0;
    // the j-th smallest column among the window's entries at key
    uint32_t cmn = 0xffffffffu, cmx = 0u;
    for (uint32_t i = tid; i < n; i += NT)
        if (wk[i] == key) { cmn = min(cmn, wc[i]); cmx = max(cmx, wc[i]); }
    cmn = block_min_u32(cmn, s);
    cmx = block_max_u32(cmx, s);
    int crem = varying_bits(cmn, cmx);
    uint32_t cpm = crem >= 32 ? 0u : ~((1u << crem) - 1u);
    uint32_t cpf = cmn & cpm;
    uint64_t crel = j;
    while (crem > 0) {
        const int w = crem < 8 ? crem : 8;
        const int shift = crem - w;
        const uint32_t dmask = (1u << w) - 1u;
        for (int b = tid; b < NB8; b += NT) cn[b] = 0u;
        __syncthreads();
        for (uint32_t i = tid; i < n; i += NT)
            if (wk[i] == key && (wc[i] & cpm) == cpf) atomicAdd(&cn[(wc[i] >> shift) & dmask], 1u);
        __syncthreads();
        if (tid < 32) scan_local(s, 1 << w, crel, false, true);
        __syncthreads();
        const SelRes r = s.ctl->sel;
        __syncthreads();
        crel -= r.before;
        cpf |= r.key << shift;
        cpm |= dmask << shift;
        crem = shift;
    }
    T.found = true;
    T.key = key;
    T.col = cpf;
    T.before_key = T.before + before;
    T.at_key = at;
    T.n_key = nat;
}

// A query: levels until every active target's bin fits the window, then the
// collection and the gather (the exact select is window_select). The filter
// is the keys in [kk, kx]; [rlo, rhi] bounds the keys the row holds. With a
// mode other than TM_FIXED, the targets are set from the first level's total
// weight Q (returned in *total).
__device__ void query(cg::cluster_group& cl, const Sm& s, int& par, int G, uint32_t ncols, uint32_t c_lo,
                      uint32_t kk, uint32_t kx, uint32_t rlo, uint32_t rhi, Tgt (&t)[2], int mode, const RowP& p,
                      float My, float scale, uint64_t* total) {
    const int tid = threadIdx.x;
    const uint32_t klo0 = max(kk, rlo), khi0 = min(kx, rhi);
    for (int tt = 0; tt < 2; ++tt) {
        t[tt].ok = false;
        t[tt].before = 0;
        t[tt].L = make_level(klo0, khi0);
        if (klo0 > khi0) t[tt].active = false;
    }
    for (int level = 0; level < 8; ++level) {
        if (!t[0].active && !t[1].active) break;
        // TM_CUT: target 1 takes target 0's first level (same filter, same range)
        const bool share = level == 0 && mode == TM_CUT && t[1].active;
        if (share) t[1].active = false;
        for (int tt = 0; tt < 2; ++tt)
            if (t[tt].active)
                for (int a = 0; a < (t[tt].mass ? 3 : 1); ++a)
                    for (int b = tid; b < NBL; b += NT) hist_ptr(s, par, tt, a)[b] = 0u;
        __syncthreads();
        const Level L0 = t[0].L, L1 = t[1].L;
        const bool a0 = t[0].active, a1 = t[1].active, m0 = t[0].mass, m1 = t[1].mass;
        for (uint32_t i = tid; i < ncols; i += NT) {
            const uint32_t k = s.cache[i];
            if (k < kk || k > kx) continue;
            const bool in0 = a0 && k >= L0.klo && k <= L0.khi;
            const bool in1 = a1 && k >= L1.klo && k <= L1.khi;
            if (!(in0 || in1)) continue;
            const uint64_t w = (m0 || m1) ? qmass(funkey(k), My, scale) : 0ull;
            if (in0) {
                const uint32_t b = bin_of(L0, k);
                atomicAdd(&hist_ptr(s, par, 0, 0)[b], 1u);
                if (m0) add_w(hist_ptr(s, par, 0, 1), hist_ptr(s, par, 0, 2), b, w);
            }
            if (in1) {
                const uint32_t b = bin_of(L1, k);
                atomicAdd(&hist_ptr(s, par, 1, 0)[b], 1u);
                if (m1) add_w(hist_ptr(s, par, 1, 1), hist_ptr(s, par, 1, 2), b, w);
            }
        }
        reduce_level(cl, s, par, G, t);
        if (level == 0 && mode != TM_FIXED) {
            // the first level sees the whole filtered set: its total weight
            unsigned long long v = 0;
            for (int b = tid; b < NBL; b += NT)
                v += ((unsigned long long)full_ptr(s, 0, 2)[b] << 32) | full_ptr(s, 0, 1)[b];
            const uint64_t Q = block_sum_u64(v, s);
            if (total) *total = Q;
            if (Q == 0) { t[0].active = false; t[1].active = false; par ^= 1; cl.sync(); break; }
            if (mode == TM_CUT) {
                t[0].target = (uint64_t)floor((double)p.top_p * (double)Q);
                t[1].target = (uint64_t)floor((double)p.u * (double)t[0].target);
                // target 1 shares target 0's first level: same filter and range
            } else {
                uint64_t dt = (uint64_t)floor((double)p.u * (double)Q);
                if (dt >= Q) dt = Q - 1;
                t[0].target = dt;
            }
        }
        if (share) {
            // target 0's reduced first level is target 1's
            t[1].active = true;
            for (int i = tid; i < 3 * NBL; i += NT) full_ptr(s, 1, 0)[i] = full_ptr(s, 0, 0)[i];
            __syncthreads();
        }
        scan_level(s, t);
        bool fits[2] = {false, false}, bigtie[2] = {false, false};
        uint32_t tbin[2] = {0u, 0u};
        for (int tt = 0; tt < 2; ++tt) {
            Tgt& T = t[tt];
            if (!T.active) continue;
            const SelRes r = s.ctl->bsel[tt];
            if (!r.ok) { T.active = false; continue; }
            T.before += r.before;
            const uint32_t blo = bin_lo_key(T.L, r.key), bhi = bin_hi_key(T.L, r.key);
            if (r.nat <= (uint32_t)WMAX) {
                fits[tt] = true;
                T.bin_at = r.at;
                T.L.klo = blo;
                T.L.khi = bhi;
            } else if (blo == bhi) {
                // one key, more ties than the window holds
                bigtie[tt] = true;
                tbin[tt] = r.key;
                T.bin_at = r.at;
                T.key = blo;
                T.n_key = r.nat;
            } else {
                T.L = make_level(blo, bhi);
            }
        }
        __syncthreads();
        if (bigtie[0] || bigtie[1]) {
            // the j-th tie (ascending column): per-CTA counts from the local
            // histograms, then the CTA that holds it scans its column-ordered
            // keys for it
            const int rank = (int)cl.block_rank();
            int owner[2] = {-1, -1};
            uint32_t jl[2] = {0u, 0u};
            for (int tt = 0; tt < 2; ++tt) {
                if (!bigtie[tt]) continue;
                Tgt& T = t[tt];
                const uint64_t rel = T.target - T.before;
                const uint64_t q = T.mass ? (T.n_key ? T.bin_at / T.n_key : 0) : 1;
                uint64_t j = q ? rel / q : 0;
                if (j >= T.n_key) j = T.n_key - 1;
                for (int qq = 0; qq < G && owner[tt] < 0; ++qq) {
                    const uint32_t nq = cl.map_shared_rank(hist_ptr(s, par, tt, 0), (unsigned)qq)[tbin[tt]];
                    if (j < nq) { owner[tt] = qq; jl[tt] = (uint32_t)j; } else j -= nq;
                }
                if (owner[tt] == rank) {
                    const uint32_t per_t = (ncols + NT - 1) / NT;
                    const uint32_t i0 = min(ncols, (uint32_t)tid * per_t), i1 = min(ncols, i0 + per_t);
                    uint32_t cnt = 0;
                    for (uint32_t i = i0; i < i1; ++i) cnt += (s.cache[i] == T.key && s.cache[i] >= kk && s.cache[i] <= kx) ? 1u : 0u;
                    // exclusive scan over the threads (column order)
                    const int lane = tid & 31, wid = tid >> 5;
                    const uint32_t incl = warp_incl_scan_u32(cnt, lane);
                    if (lane == 31) s.ctl->red32[wid] = incl;
                    __syncthreads();
                    uint32_t base = 0;
                    for (int w2 = 0; w2 < wid; ++w2) base += s.ctl->red32[w2];
                    base += incl - cnt;
                    if (jl[tt] >= base && jl[tt] < base + cnt) {
                        uint32_t need = jl[tt] - base;
                        for (uint32_t i = i0; i < i1; ++i) {
                            if (s.cache[i] == T.key) {
                                if (need == 0) { s.ctl->tiecol[tt] = c_lo + i; break; }
                                --need;
                            }
                        }
                    }
                    __syncthreads();
                }
            }
            cl.sync();
            for (int tt = 0; tt < 2; ++tt) {
                if (!bigtie[tt]) continue;
                Tgt& T = t[tt];
                T.col = owner[tt] >= 0 ? *cl.map_shared_rank(&s.ctl->tiecol[tt], (unsigned)owner[tt]) : 0xffffffffu;
                T.found = owner[tt] >= 0;
                T.ok = T.found;
                T.before_key = T.before;
                T.at_key = T.bin_at;
                T.active = false;
            }
        }
        if (!fits[0] && !fits[1]) { par ^= 1; continue; }
        // collect this CTA's elements of each fitting bin, then gather every CTA's list
        if (tid < 2) s.ctl->wcnt[tid] = 0u;
        __syncthreads();
        const Level F0 = t[0].L, F1 = t[1].L;
        for (uint32_t i = tid; i < ncols; i += NT) {
            const uint32_t k = s.cache[i];
            if (k < kk || k > kx) continue;
            if (fits[0] && k >= F0.klo && k <= F0.khi) {
                const uint32_t pos = atomicAdd(&s.ctl->wcnt[0], 1u);
                if (pos < (uint32_t)WMAX) { wloc_ptr(s, 0, 0)[pos] = k; wloc_ptr(s, 0, 1)[pos] = c_lo + i; }
            }
            if (fits[1] && k >= F1.klo && k <= F1.khi) {
                const uint32_t pos = atomicAdd(&s.ctl->wcnt[1], 1u);
                if (pos < (uint32_t)WMAX) { wloc_ptr(s, 1, 0)[pos] = k; wloc_ptr(s, 1, 1)[pos] = c_lo + i; }
            }
        }
        __syncthreads();
        if (tid == 0) {
            Part& pt = s.ctl->part[par];
            pt.nloc[0] = min(s.ctl->wcnt[0], (uint32_t)WMAX);
            pt.nloc[1] = min(s.ctl->wcnt[1], (uint32_t)WMAX);
        }
        cl.sync();
        for (int tt = 0; tt < 2; ++tt) {
            if (!fits[tt]) continue;
            uint32_t off = 0;
            for (int q = 0; q < G; ++q) {
                const uint32_t nq = cl.map_shared_rank(&s.ctl->part[par], (unsigned)q)->nloc[tt];
                const uint32_t* rk = cl.map_shared_rank(wloc_ptr(s, tt, 0), (unsigned)q);
                const uint32_t* rc = cl.map_shared_rank(wloc_ptr(s, tt, 1), (unsigned)q);
                for (uint32_t i = tid; i < nq && off + i < (uint32_t)WMAX; i += NT) {
                    wall_ptr(s, tt, 0)[off + i] = rk[i];
                    wall_ptr(s, tt, 1)[off + i] = rc[i];
                }
                off += nq;
            }
            t[tt].n = min(off, (uint32_t)WMAX);
            t[tt].ok = true;
            t[tt].gathered = true;
            t[tt].active = false;
        }
        par ^= 1;
        // the peers read this CTA's lists: keep them until every CTA is done
        cl.sync();
    }
    t[0].active = false;
    t[1].active = false;
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(NT, 1) cluster_kernel(const __grid_constant__ Params P) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE;
    constexpr int VEC = E::VEC;
    cg::cluster_group cl = cg::this_cluster();
    const int rank = (int)cl.block_rank();
    const int G = (int)cl.num_blocks();
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    const float scale = __uint_as_float((uint32_t)(127 + P.mass_shift) << 23);   // 2^S
    const unsigned B = (unsigned)P.batch;
    for (int i = tid; i < P.swords; i += NT) s.bitmap[i] = 0u;
    if (tid == 0) { s.ctl->npend = 0u; s.ctl->pend_mask = 0u; s.ctl->pend_base = 0u; }
    __syncthreads();
    int par = 0;   // exchange-buffer parity

    for (;;) {
        // ---- claim a row (warp 0 of rank 0), publish it to the cluster ----
        // Every row when all_rows; otherwise rows are claimed in chunks and
        // the deferred ones among them found with one ballot per chunk.
        if (rank == 0 && tid < 32) {
            const unsigned chunk = P.all_rows ? 1u : (unsigned)CLAIM_CHUNK;
            while (s.ctl->npend == 0u) {
                unsigned v = 0;
                if (tid == 0) v = atomicAdd(&P.ws[2], chunk);
                v = __shfl_sync(0xffffffffu, v, 0);
                if (v >= B) break;
                const unsigned rr = v + (unsigned)tid;
                const bool want = tid < (int)chunk && rr < B && (P.all_rows || __ldcg(P.out_ids + rr) == kDeferredId);
                const uint32_t bal = __ballot_sync(0xffffffffu, want);
                if (tid == 0) { s.ctl->pend_base = v; s.ctl->pend_mask = bal; s.ctl->npend = __popc(bal); }
                __syncwarp();
            }
            __syncwarp();
            if (tid == 0) {
                int r = -1;
                if (s.ctl->npend > 0u) {
                    const uint32_t m = s.ctl->pend_mask;
                    r = (int)(s.ctl->pend_base + (unsigned)(__ffs(m) - 1));
                    s.ctl->pend_mask = m & (m - 1u);
                    s.ctl->npend -= 1u;
                }
                s.ctl->row = r;
            }
        }
        cl.sync();
        const int r = *cl.map_shared_rank(&s.ctl->row, 0u);
        if (r < 0) break;

        const bool has_hist = P.pen_possible && (__ldg(P.hist_offsets + r + 1) > __ldg(P.hist_offsets + r));
        const RowP p = load_row_params(P.temperature, P.top_p, P.top_k, P.rep, P.pres, P.freq, P.greedy, P.uniforms, r,
                                       has_hist, P.vocab);
        const Geom g = row_geom<ESZ>(P.logits, P.row_stride, P.vocab, r);
        const Slice sl = make_slice<ESZ>(g, P.vocab, rank, G);
        const uint32_t ncols = (uint32_t)(sl.c_hi - sl.c_lo);
        uint32_t* flags = &s.ctl->wcnt[0];
        if (tid == 0) *flags = 0u;
        __syncthreads();
        const uint32_t U = p.pen ? slice_history<DT>(P, s, g, sl, p, r, flags) : 0u;
        const uint32_t lflags = *flags;
        __syncthreads();

        // ---- pass 1: penalties, y = x / T, key cache; maximum, first argmax, first NaN ----
        float mx = -INFINITY, bv = -INFINITY;
        uint32_t bc = 0xffffffffu, nanc = 0xffffffffu, kmin = 0xffffffffu;
        auto take = [&](float x, uint32_t c) {
            mx = fmax_nan(mx, x);
            if (arg_better(x, c, bv, bc)) { bv = x; bc = c; }
            if (x != x) nanc = min(nanc, c);
            const uint32_t k = fkey(ydiv(p, x));
            kmin = min(kmin, k);
            s.cache[c - (uint32_t)sl.c_lo] = k;
        };
        {
            const uint4* src = reinterpret_cast<const uint4*>(g.interior) + sl.ch0;
            const int n = sl.ch1 - sl.ch0;
            const bool pen = p.pen;
            auto chunk = [&](const uint4& v, int i) {
                const int c0 = g.head + (sl.ch0 + i) * VEC;
                float x[VEC];
                E::unpack(v, x);
                uint32_t hb = 0u;
                if (pen) {
                    const int o = c0 - sl.c_lo;
                    const int w = o >> 5, b = o & 31;
                    const uint32_t lo = s.bitmap[w];
                    const uint32_t hi = (b + VEC > 32 && w + 1 < P.swords) ? s.bitmap[w + 1] : 0u;
                    hb = __funnelshift_r(lo, hi, b) & ((1u << VEC) - 1u);
                }
#pragma unroll
                for (int e = 0; e < VEC; ++e)
                    if (!((hb >> e) & 1u)) take(x[e], (uint32_t)(c0 + e));
            };
            constexpr int U4 = 4;
            int i = tid;
            for (; i + (U4 - 1) * NT < n; i += U4 * NT) {
                uint4 v[U4];
#pragma unroll
                for (int j = 0; j < U4; ++j) v[j] = __ldg(src + i + j * NT);
#pragma unroll
                for (int j = 0; j < U4; ++j) chunk(v[j], i + j * NT);
            }
            for (; i < n; i += NT) chunk(__ldg(src + i), i);
            // ragged head / tail columns (fewer than VEC each)
            const int nh = sl.head ? g.head : 0;
            const int nt = sl.tail ? (P.vocab - g.tail0) : 0;
            if (tid < nh + nt) {
                const int c = tid < nh ? tid : g.tail0 + (tid - nh);
                if (c >= sl.c_lo && c < sl.c_hi) {
                    const int o = c - sl.c_lo;
                    const bool hist = pen && ((s.bitmap[o >> 5] >> (o & 31)) & 1u);
                    if (!hist) take(E::load(g.row, c), (uint32_t)c);
                }
            }
            for (uint32_t h = tid; h < U; h += NT) take(s.hval[h], s.hcol[h]);
        }
        mx = block_max_nan(mx, s);
        block_argmax(bv, bc, s);
        nanc = block_min_u32(nanc, s);
        kmin = block_min_u32(kmin, s);
        if (tid == 0) {
            Part& pt = s.ctl->part[par];
            pt.mx = mx; pt.bv = bv; pt.bc = bc; pt.nan_col = nanc; pt.flags = lflags; pt.pad = kmin;
        }
        cl.sync();
        float M = -INFINITY;
        float gbv = -INFINITY;
        uint32_t gbc = 0xffffffffu, gnan = 0xffffffffu, gflags = 0u, gkmin = 0xffffffffu;
        for (int q = 0; q < G; ++q) {
            const Part* pt = cl.map_shared_rank(&s.ctl->part[par], (unsigned)q);
            M = fmax_nan(M, pt->mx);
            if (arg_better(pt->bv, pt->bc, gbv, gbc)) { gbv = pt->bv; gbc = pt->bc; }
            gnan = min(gnan, pt->nan_col);
            gflags |= pt->flags;
            gkmin = min(gkmin, pt->pad);
        }
        par ^= 1;

        int status = p.bad | (int)gflags | FG_ROW_GENERAL_PATH;
        int64_t out = -1;
        // kept set: key >= ykK and, with a cut, (key > tstar or (key == tstar
        // and column <= id_cut))
        uint32_t ykK = 0u, tstar = 0u, id_cut = 0xffffffffu;
        bool cut = false, sampled = false;
        uint64_t Qf = 0;
        float My = 0.0f;

        if (status & (FG_ROW_BAD_PARAM | FG_ROW_BAD_UNIFORM)) {
            out = -1;
        } else if (p.cls == RC_GREEDY) {
            status |= FG_ROW_GREEDY;
            out = (M != M) ? (int64_t)gnan : (int64_t)gbc;
        } else if (M != M) {
            status |= FG_ROW_NAN;
        } else if (M == INFINITY) {
            status |= FG_ROW_POS_INF;
        } else if (M == -INFINITY) {
            status |= FG_ROW_ALL_MASKED;
        } else {
            My = ydiv(p, M);
            const uint32_t rlo = gkmin, rhi = fkey(My);
            const uint32_t c_lo = (uint32_t)sl.c_lo;
            // ---- top-k threshold: the K-th largest key by count ----
            if (p.cls == RC_TOPK && p.K < P.vocab) {
                Tgt t[2] = {tgt(true, false, (uint64_t)(p.K - 1)), tgt(false, false, 0)};
                query(cl, s, par, G, ncols, c_lo, 0u, 0xffffffffu, rlo, rhi, t, TM_FIXED, p, My, scale, nullptr);
                if (t[0].gathered) window_select(s, 0, t[0].target - t[0].before, My, scale, t[0]);
                ykK = t[0].found ? t[0].key : 0u;
            }
            // ---- top-p cut and the draw: mass queries over the kept set ----
            uint64_t Q = 0;
            uint32_t dcol = 0u;
            bool drawn = false;
            if (p.use_p) {
                // target 0: the cut at floor(top_p * Q); target 1: the draw
                // predicted from it (the kept mass exceeds the cut's target by
                // less than one element's mass, so the draw's target lies
                // within a bin of the prediction's, mostly the same bin)
                Tgt t[2] = {tgt(true, true, 0), tgt(true, true, 0)};
                query(cl, s, par, G, ncols, c_lo, ykK, 0xffffffffu, rlo, rhi, t, TM_CUT, p, My, scale, &Q);
                if (t[0].gathered) window_select(s, 0, t[0].target - t[0].before, My, scale, t[0]);
                if (t[0].found) {
                    cut = true;
                    tstar = t[0].key;
                    const uint64_t qt = t[0].n_key ? t[0].at_key / t[0].n_key : 0;
                    uint64_t m = t[0].n_key;
                    if (qt > 0) {
                        const uint64_t mm = (t[0].target - t[0].before_key) / qt + 1;
                        if (mm < m) m = mm;
                    }
                    Qf = t[0].before_key + m * qt;
                    uint64_t Dt = (uint64_t)floor((double)p.u * (double)Qf);
                    if (Dt >= Qf) Dt = Qf - 1;
                    // the element at Dt in descending order lies in the cut's kept
                    // part (Dt < Qf), so the unrestricted order finds it
                    if (t[1].gathered && Dt >= t[1].before && Dt < t[1].before + t[1].bin_at) {
                        t[1].target = Dt;
                        window_select(s, 1, Dt - t[1].before, My, scale, t[1]);
                        if (t[1].found) { dcol = t[1].col; drawn = true; }
                    }
                    if (!drawn) {
                        Tgt d[2] = {tgt(true, true, Dt), tgt(false, true, 0)};
                        query(cl, s, par, G, ncols, c_lo, ykK, 0xffffffffu, rlo, rhi, d, TM_FIXED, p, My, scale, nullptr);
                        if (d[0].gathered) window_select(s, 0, Dt - d[0].before, My, scale, d[0]);
                        if (d[0].found) { dcol = d[0].col; drawn = true; }
                    }
                    if (P.out_probs != nullptr && m < t[0].n_key) {
                        // the last kept tie at the cut: the m-th (ascending column) at tstar
                        Tgt c[2] = {tgt(true, false, m - 1), tgt(false, false, 0)};
                        query(cl, s, par, G, ncols, c_lo, tstar, tstar, rlo, rhi, c, TM_FIXED, p, My, scale, nullptr);
                        if (c[0].gathered) window_select(s, 0, c[0].target - c[0].before, My, scale, c[0]);
                        id_cut = c[0].found ? c[0].col : 0xffffffffu;
                    }
                }
            } else {
                Tgt t[2] = {tgt(true, true, 0), tgt(false, true, 0)};
                query(cl, s, par, G, ncols, c_lo, ykK, 0xffffffffu, rlo, rhi, t, TM_DRAW, p, My, scale, &Q);
                Qf = Q;
                if (t[0].gathered) window_select(s, 0, t[0].target - t[0].before, My, scale, t[0]);
                if (t[0].found) { dcol = t[0].col; drawn = true; }
            }
            if (drawn) { out = (int64_t)dcol; sampled = true; }
            if (out < 0 && !(status & FG_ROW_ERROR_MASK)) status |= FG_ROW_ALL_MASKED;
        }
        // ---- kept-set probabilities (debug / oracle mode) ----
        if (P.out_probs != nullptr) {
            float* pr = P.out_probs + (int64_t)r * P.vocab;
            const double inv = (sampled && Qf > 0) ? 1.0 / (double)Qf : 0.0;
            const bool greedy_row = p.cls == RC_GREEDY && out >= 0;
            for (uint32_t i = tid; i < ncols; i += NT) {
                const uint32_t c = (uint32_t)sl.c_lo + i;
                float v = 0.0f;
                if (greedy_row) {
                    v = (c == (uint32_t)out) ? 1.0f : 0.0f;
                } else if (sampled) {
                    const uint32_t k = s.cache[i];
                    bool keep = k >= ykK;
                    if (keep && cut) keep = k > tstar || (k == tstar && c <= id_cut);
                    if (keep) v = (float)((double)qmass(funkey(k), My, scale) * inv);
                }
                pr[c] = v;
            }
        }
        // ---- outputs ----
        if (rank == 0 && tid == 0) {
            P.out_ids[r] = out >= 0 ? out + P.vocab_offset : -1;
            if (P.out_status) P.out_status[r] = status;
        }
        // clear this row's slice bitmap bits for the next row (all of it if
        // the history table lost columns)
        if (p.pen && s.ctl->nuniq > U) {
            for (int i = tid; i < P.swords; i += NT) s.bitmap[i] = 0u;
        } else {
            for (uint32_t i = tid; i < U; i += NT) {
                const int o = (int)s.hcol[i] - sl.c_lo;
                s.bitmap[o >> 5] = 0u;
            }
        }
        __syncthreads();
    }
    // ---- the last cluster leaves the claim counters zero ----
    cl.sync();
    if (rank == 0 && tid == 0) {
        __threadfence();
        const unsigned ncl = gridDim.x / (unsigned)G;
        if (atomicAdd(&P.ws[3], 1u) == ncl - 1u) {
            P.ws[2] = 0u;
            P.ws[3] = 0u;
            __threadfence();
        }
    }
}

}  // namespace clus
}  // namespace fg
