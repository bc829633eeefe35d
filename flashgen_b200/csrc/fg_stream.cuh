// fg_stream.cuh — the batch path of fg_sample (sm_100a): three kernels per call.
//
//   K1 prep_kernel     one CTA per row with penalties: the row's distinct history
//                      columns with their counts, written to the row's
//                      workspace block (K2 gathers their raw logits right after
//                      streaming the row, from L2, and writes their penalised
//                      values: FlashGen's repetition penalty, plus presence and
//                      frequency; their best value and NaN-propagating maximum).
//   K2 stream_kernel   persistent CTAs, two per SM, each a producer warp and
//                      NCW consumer warps. The producer takes rows from a global
//                      queue (rows that sum exp over the whole row first) and
//                      streams each row's 16-byte-aligned interior HBM -> shared
//                      memory through a ring of 16 KB stages with 1-D bulk async
//                      copies (cp.async.bulk, completion on mbarriers), claiming
//                      the next row as soon as the current row's last copy is
//                      issued. A penalised row's history columns are set in a
//                      shared-memory column bitmap and masked to -inf chunk by
//                      chunk. Over the remaining columns the consumers keep a
//                      packed NaN-propagating maximum, and by row class the first
//                      argmax (greedy rows, finished here), an online sum of exp
//                      (top-k off), and a candidate filter x >= tau that appends
//                      (key, column) to a shared buffer. tau starts from the
//                      tile-0 chunk maxima and rises with one-pass compactions of
//                      the buffer. At the row's end the buffer and the row's
//                      statistics go to the row's workspace block: the next
//                      row's tiles are already in the ring.
//   K3 decide_kernel   one small CTA per remaining row: the candidates plus the
//                      penalised history entries at or above tau, the sum of exp
//                      of the non-history columns plus the history columns'
//                      penalised terms, then the exact K-th largest, top-p cut
//                      and draw (integer masses, radix selects). A row the
//                      candidates cannot decide is handed to the cluster kernel
//                      (fg_cluster.cuh): out_ids = kDeferredId.
//
// Reference: flashgen/sampling/sampler.py:57-169; draw order of
// csrc/runtime/pipeline.cpp:311-340.
#pragma once

#include "fg_row.cuh"

namespace fg {
namespace strm {

constexpr int NCW = 8;                  // consumer warps
constexpr int NCT = NCW * 32;           // consumer threads
constexpr int NTH = NCT + 32;           // + producer warp
constexpr int TILE = 16384;             // ring stage bytes
constexpr int CPT = TILE / 16 / NCT;    // 16-byte chunks per consumer thread per tile
constexpr int RQ = 2;                   // row-queue slots
constexpr int NB = 256;                 // radix bins
constexpr int BAR = 1;                  // named barrier of the consumer warps
constexpr uint32_t kSkip = 0x80000000u; // row-queue flag: the row is not streamed
constexpr int64_t kPendingId = -3;      // out_ids of a row K2 leaves to K3
constexpr int64_t kDeepId = -4;         // out_ids of a row K3 leaves to K4

// Per-row workspace block (16-byte aligned parts):
//   RowStat, HistHdr, hcol[hu_cap], hcnt[hu_cap], hpen[hu_cap], ckey[cap], ccol[cap]
struct RowStat {
    double zr;        // sum over the raw row of 2^((x - mraw) * c)
    float mraw;       // NaN-propagating maximum of the raw row
    float tau;        // the candidates are complete above tau (penalised, non-history)
    uint32_t n;       // candidates
    uint32_t ovf;     // the buffer overflowed: incomplete
    uint32_t pad[2];
    // K3 -> K4 (rows whose cut or draw lies below the candidates)
    double zq;        // the row's total mass (mass units, from the sums of exp)
    unsigned long long ac;   // exact mass of the candidate set
    float mfin;       // the row's maximum after penalties
    uint32_t pad2[3];
};
struct HistHdr {
    uint32_t nh;      // distinct history columns kept (<= hu_cap)
    uint32_t flags;   // FG_ROW_BAD_HISTORY / FG_ROW_BAD_PARAM
    float pbest;      // best penalised history value and its first column (K2)
    uint32_t pcol;
    float hmax;       // NaN-propagating maximum of the penalised history values (K2)
    uint32_t pad[3];
};
__host__ __device__ inline int64_t wrow_bytes(int hu_cap, int cap) {
    return (int64_t)sizeof(RowStat) + (int64_t)sizeof(HistHdr) + 12ll * ((hu_cap + 3) / 4 * 4) + 8ll * cap;
}

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
    unsigned int* ws;          // [0] queue position, [1] finished CTAs
    uint8_t* wrow;             // per-row blocks
    int64_t wrow_bytes;
    int32_t nstage;
    int32_t cap;               // candidate buffer entries (shared memory and row block)
    int32_t k_fast;            // largest top-k decided from the candidates
    int32_t k_nuc;             // candidate target of rows with top-k off
    int32_t hu_cap;            // history table entries (0: no penalties in this call)
    int32_t hcap4;             // hu_cap rounded up to 4
    int32_t hslots;            // K1: hash slots (power of two >= 2 * hu_cap)
    int32_t nwords;            // K2: history bitmap words (columns / 32, rounded up)
    int32_t pen_possible;
    int32_t mass_shift;
    int32_t off_ctl, off_bins, off_ckey, off_ccol, off_hbm, off_ring;
    int32_t off_cnt, off_tsum, off_hl;   // K4: key counts, per-thread masses, history entries
};

// Parts of row r's workspace block.
__device__ __forceinline__ RowStat* row_stat(const Params& P, int r) {
    return reinterpret_cast<RowStat*>(P.wrow + (int64_t)r * P.wrow_bytes);
}
__device__ __forceinline__ HistHdr* hist_hdr(const Params& P, int r) {
    return reinterpret_cast<HistHdr*>(P.wrow + (int64_t)r * P.wrow_bytes + sizeof(RowStat));
}
__device__ __forceinline__ uint32_t* g_hcol(const Params& P, int r) {
    return reinterpret_cast<uint32_t*>(P.wrow + (int64_t)r * P.wrow_bytes + sizeof(RowStat) + sizeof(HistHdr));
}
__device__ __forceinline__ uint32_t* g_hcnt(const Params& P, int r) { return g_hcol(P, r) + P.hcap4; }
__device__ __forceinline__ float* g_hpen(const Params& P, int r) {
    return reinterpret_cast<float*>(g_hcol(P, r) + 2 * P.hcap4);
}
__device__ __forceinline__ uint32_t* g_ckey(const Params& P, int r) { return g_hcol(P, r) + 3 * P.hcap4; }
__device__ __forceinline__ uint32_t* g_ccol(const Params& P, int r) { return g_ckey(P, r) + P.cap; }

struct SelRes {
    uint32_t key;
    uint32_t ok;
    uint32_t nat;
    uint32_t pad;
    unsigned long long before, at;
};

struct Ctl {
    uint32_t rowq[RQ];
    int abort;
    int status;
    uint32_t ncand;
    uint32_t ovf;
    uint32_t nuniq;
    uint32_t snap;
    float tau;
    uint32_t b32[4];
    SelRes sel;
    float redf[NCW];
    uint32_t red32[NCW];
    uint32_t red32b[NCW];
    unsigned long long red64[NCW];
    double redd[NCW];
};

extern __shared__ __align__(128) uint8_t ssmem[];

struct Sm {
    uint64_t* full;
    uint64_t* empty;
    uint64_t* rfull;
    uint64_t* rempty;
    Ctl* ctl;
    uint32_t* bcnt;   // [NB]
    uint32_t* blo;    // [NB]
    uint32_t* bhi;    // [NB]
    uint32_t* ckey;
    uint32_t* ccol;
    uint32_t* hbm;    // K2: bitmap of the row's history columns (nwords + 1 words)
    uint8_t* ring;
};
__host__ __device__ inline int bar_bytes(int ns) { return 8 * (2 * ns + 2 * RQ); }
__device__ __forceinline__ Sm carve(const Params& P) {
    Sm s;
    s.full = reinterpret_cast<uint64_t*>(ssmem);
    s.empty = s.full + P.nstage;
    s.rfull = s.empty + P.nstage;
    s.rempty = s.rfull + RQ;
    s.ctl = reinterpret_cast<Ctl*>(ssmem + P.off_ctl);
    s.bcnt = reinterpret_cast<uint32_t*>(ssmem + P.off_bins);
    s.blo = s.bcnt + NB;
    s.bhi = s.blo + NB;
    s.ckey = reinterpret_cast<uint32_t*>(ssmem + P.off_ckey);
    s.ccol = reinterpret_cast<uint32_t*>(ssmem + P.off_ccol);
    s.hbm = reinterpret_cast<uint32_t*>(ssmem + P.off_hbm);
    s.ring = ssmem + P.off_ring;
    return s;
}

// ---------------------------------------------------------------------------
// Consumer-group reductions (named barrier BAR, NCT threads)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void csync() { named_sync(BAR, NCT); }

// ---------------------------------------------------------------------------
// Consumer-group reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float c_max_nan(float v, const Sm& s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s.ctl->redf[w] = v;
    csync();
    float r = s.ctl->redf[0];
#pragma unroll
    for (int i = 1; i < NCW; ++i) r = fmax_nan(r, s.ctl->redf[i]);
    csync();
    return r;
}
__device__ __forceinline__ uint32_t c_sum_u32(uint32_t v, const Sm& s) {
    v = __reduce_add_sync(0xffffffffu, v);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s.ctl->red32[w] = v;
    csync();
    uint32_t r = 0;
#pragma unroll
    for (int i = 0; i < NCW; ++i) r += s.ctl->red32[i];
    csync();
    return r;
}
__device__ __forceinline__ void c_minmax_u32(uint32_t& mn, uint32_t& mx, const Sm& s) {
    mn = __reduce_min_sync(0xffffffffu, mn);
    mx = __reduce_max_sync(0xffffffffu, mx);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { s.ctl->red32[w] = mn; s.ctl->red32b[w] = mx; }
    csync();
    uint32_t a = s.ctl->red32[0], b = s.ctl->red32b[0];
#pragma unroll
    for (int i = 1; i < NCW; ++i) { a = min(a, s.ctl->red32[i]); b = max(b, s.ctl->red32b[i]); }
    csync();
    mn = a;
    mx = b;
}
__device__ __forceinline__ unsigned long long c_sum_u64(unsigned long long v, const Sm& s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += shfl_u64(v, (threadIdx.x & 31) ^ o);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s.ctl->red64[w] = v;
    csync();
    unsigned long long r = 0;
#pragma unroll
    for (int i = 0; i < NCW; ++i) r += s.ctl->red64[i];
    csync();
    return r;
}
// Deterministic double sum: fixed shuffle tree, then warps in index order.
__device__ __forceinline__ double c_sum_f64(double v, const Sm& s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s.ctl->redd[w] = v;
    csync();
    double r = 0.0;
#pragma unroll
    for (int i = 0; i < NCW; ++i) r += s.ctl->redd[i];
    csync();
    return r;
}
__device__ __forceinline__ bool arg_better(float v, uint32_t c, float v2, uint32_t c2) {
    return v > v2 || (v == v2 && c < c2);
}
__device__ __forceinline__ void c_argmax(float& v, uint32_t& c, const Sm& s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t c2 = __shfl_xor_sync(0xffffffffu, c, o);
        if (arg_better(v2, c2, v, c)) { v = v2; c = c2; }
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { s.ctl->redf[w] = v; s.ctl->red32[w] = c; }
    csync();
    float bv = s.ctl->redf[0];
    uint32_t bc = s.ctl->red32[0];
#pragma unroll
    for (int i = 1; i < NCW; ++i)
        if (arg_better(s.ctl->redf[i], s.ctl->red32[i], bv, bc)) { bv = s.ctl->redf[i]; bc = s.ctl->red32[i]; }
    csync();
    v = bv;
    c = bc;
}

// ---------------------------------------------------------------------------
// Radix select (descending keys) over weights that every consumer thread
// yields through enumerate(f): f(valid, key, weight), called the same number
// of times in every lane of a warp. Finds the key k* with
//     W(keys > k*) <= target < W(keys >= k*)
// among keys in [klo, khi]. Exact integer weights (counts when !MASS).
// ---------------------------------------------------------------------------
struct Sel {
    uint32_t key;
    uint64_t before, at;
    uint32_t nat;
    bool ok;
};
__device__ __forceinline__ int varying_bits(uint32_t lo, uint32_t hi) {
    const uint32_t d = lo ^ hi;
    return d == 0 ? 0 : 32 - __clz(d);
}
// Warp 0: the digit of nb (<= NB) bins, scanned in descending order, that
// holds `rel`.
template <bool MASS>
__device__ __forceinline__ void scan_desc(const Sm& s, int nb, uint64_t rel) {
    const int lane = threadIdx.x & 31;
    uint64_t v[8];
    uint64_t lsum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int o = lane * 8 + j;
        const int d = nb - 1 - o;
        v[j] = (o < nb) ? (MASS ? (((uint64_t)s.bhi[d] << 32) | s.blo[d]) : (uint64_t)s.bcnt[d]) : 0ull;
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
        const int d = nb - 1 - (lane * 8 + jj);
        o.ok = 1u;
        o.key = (uint32_t)d;
        o.before = c;
        o.nat = s.bcnt[d];
        o.at = MASS ? (((uint64_t)s.bhi[d] << 32) | s.blo[d]) : (uint64_t)s.bcnt[d];
    }
}
template <bool MASS, class Enum>
__device__ Sel c_select(const Sm& s, Enum&& enumerate, uint64_t target, uint32_t klo, uint32_t khi) {
    const int tid = threadIdx.x;
    Sel out;
    out.ok = false; out.key = 0u; out.before = 0; out.at = 0; out.nat = 0u;
    if (klo > khi) return out;
    int rem = varying_bits(klo, khi);
    uint32_t pmask = rem >= 32 ? 0u : ~((1u << rem) - 1u);
    uint32_t prefix = klo & pmask;
    uint64_t before = 0;
    if (rem == 0) {
        // a single key: its weight
        uint64_t w = 0, n = 0;
        enumerate([&](bool valid, uint32_t k, uint64_t wt) {
            if (valid && k == prefix) { ++n; w += MASS ? wt : 1ull; }
        });
        const uint64_t W = c_sum_u64(w, s);
        const uint64_t N = MASS ? c_sum_u64(n, s) : W;
        out.ok = target < W; out.key = prefix; out.before = 0; out.at = W; out.nat = (uint32_t)N;
        return out;
    }
    while (rem > 0) {
        const int w = rem < 8 ? rem : 8;
        const int shift = rem - w;
        const uint32_t dmask = (1u << w) - 1u;
        for (int b = tid; b < NB; b += NCT) { s.bcnt[b] = 0u; s.blo[b] = 0u; s.bhi[b] = 0u; }
        csync();
        const uint32_t pm = pmask, pf = prefix;
        enumerate([&](bool valid, uint32_t k, uint64_t wt) {
            if (!valid || (k & pm) != pf) return;
            const uint32_t d = (k >> shift) & dmask;
            atomicAdd(&s.bcnt[d], 1u);
            if (MASS && wt) {
                const uint32_t l = (uint32_t)wt;
                uint32_t h = (uint32_t)(wt >> 32);
                if (l) {
                    const uint32_t old = atomicAdd(&s.blo[d], l);
                    h += (old + l < old) ? 1u : 0u;
                }
                if (h) atomicAdd(&s.bhi[d], h);
            }
        });
        csync();
        if (tid < 32) scan_desc<MASS>(s, 1 << w, target - before);
        csync();
        const SelRes r = s.ctl->sel;
        csync();
        if (!r.ok) return out;
        before += r.before;
        prefix |= r.key << shift;
        pmask |= dmask << shift;
        rem = shift;
        out.at = r.at;
        out.nat = r.nat;
    }
    out.ok = true;
    out.key = prefix;
    out.before = before;
    return out;
}

// ---------------------------------------------------------------------------
// Chunk helpers (one 16-byte chunk = VEC elements)
// ---------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ float elem_at(const uint4& v, int e) {
    if constexpr (DT == FG_DTYPE_F32) {
        return __uint_as_float(e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w);
    } else {
        const int q = e >> 1;
        const uint32_t ww = q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w;
        const uint16_t h = (e & 1) ? (uint16_t)(ww >> 16) : (uint16_t)(ww & 0xffffu);
        if constexpr (DT == FG_DTYPE_BF16) return __uint_as_float(uint32_t(h) << 16);
        else return __half2float(__ushort_as_half(h));
    }
}
// NaN-propagating maximum of a chunk (packed pairs for the 16-bit types).
template <int DT>
__device__ __forceinline__ float chunk_max(const uint4& v) {
    if constexpr (DT == FG_DTYPE_F32) {
        return fmax_nan(fmax_nan(__uint_as_float(v.x), __uint_as_float(v.y)),
                        fmax_nan(__uint_as_float(v.z), __uint_as_float(v.w)));
    } else if constexpr (DT == FG_DTYPE_BF16) {
        const __nv_bfloat162 a = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162*>(&v.x),
                                             *reinterpret_cast<const __nv_bfloat162*>(&v.y));
        const __nv_bfloat162 b = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162*>(&v.z),
                                             *reinterpret_cast<const __nv_bfloat162*>(&v.w));
        const __nv_bfloat162 m = __hmax2_nan(a, b);
        return fmax_nan(__low2float(m), __high2float(m));
    } else {
        const __half2 a = __hmax2_nan(*reinterpret_cast<const __half2*>(&v.x), *reinterpret_cast<const __half2*>(&v.y));
        const __half2 b = __hmax2_nan(*reinterpret_cast<const __half2*>(&v.z), *reinterpret_cast<const __half2*>(&v.w));
        const __half2 m = __hmax2_nan(a, b);
        return fmax_nan(__low2float(m), __high2float(m));
    }
}
// Element e of a chunk set to -inf (selects on the four words, so the chunk
// stays in registers).
template <int DT>
__device__ __forceinline__ void elem_mask_inf(uint4& v, int e) {
    if constexpr (DT == FG_DTYPE_F32) {
        constexpr uint32_t W = 0xFF800000u;
        v.x = e == 0 ? W : v.x; v.y = e == 1 ? W : v.y; v.z = e == 2 ? W : v.z; v.w = e == 3 ? W : v.w;
    } else {
        constexpr uint32_t W = DT == FG_DTYPE_BF16 ? 0xFF80FF80u : 0xFC00FC00u;
        const int q = e >> 1;
        const uint32_t keep = (e & 1) ? 0x0000ffffu : 0xffff0000u;
        const uint32_t neg = W & ~keep;
        v.x = q == 0 ? ((v.x & keep) | neg) : v.x;
        v.y = q == 1 ? ((v.y & keep) | neg) : v.y;
        v.z = q == 2 ? ((v.z & keep) | neg) : v.z;
        v.w = q == 3 ? ((v.w & keep) | neg) : v.w;
    }
}

// History bits of the VEC columns [c0, c0 + VEC) (bit e: column c0 + e), from
// the row's column bitmap (one word past the last column is kept zero).
template <int VEC>
__device__ __forceinline__ uint32_t hist_bits(const uint32_t* bm, uint32_t c0) {
    const uint32_t w = c0 >> 5, b = c0 & 31u;
    uint32_t x = bm[w] >> b;
    if (b + VEC > 32u) x |= bm[w + 1] << (32u - b);
    return x & ((1u << VEC) - 1u);
}
__device__ __forceinline__ bool hist_bit(const uint32_t* bm, uint32_t c) { return (bm[c >> 5] >> (c & 31u)) & 1u; }

// ===========================================================================
// K1: history of every row with penalties
// ===========================================================================
// Distinct history columns with their counts (open-addressed hash; the work
// follows the history, not the vocabulary). No logit is read here: a scattered
// gather would pull a whole line from HBM per column, while K2 finds the row
// in L2 right after streaming it.
template <int DT>
__global__ void __launch_bounds__(NCT) prep_kernel(const __grid_constant__ Params P) {
    using E = Elem<DT>;
    const int r = blockIdx.x;
    const int tid = threadIdx.x;
    const Sm s = carve(P);
    HistHdr* hh = hist_hdr(P, r);
    const bool has_hist = __ldg(P.hist_offsets + r + 1) > __ldg(P.hist_offsets + r);
    const RowP p = load_row_params(P.temperature, P.top_p, P.top_k, P.rep, P.pres, P.freq, P.greedy, P.uniforms, r,
                                   has_hist, P.vocab);
    if (!p.pen) {
        if (tid == 0) { hh->nh = 0u; hh->flags = 0u; hh->pbest = -INFINITY; hh->pcol = 0xffffffffu; hh->hmax = -INFINITY; }
        return;
    }
    // shared memory: the count hash, then the distinct columns (sort buffer)
    uint32_t* hkey = reinterpret_cast<uint32_t*>(ssmem + P.off_ctl + sizeof(Ctl));
    uint32_t* hcnt = hkey + P.hslots;
    uint32_t* srt = hcnt + P.hslots;          // hslots / 2 >= hu_cap entries (a power of two)
    Ctl* ctl = s.ctl;
    const uint32_t mask = (uint32_t)P.hslots - 1u;
    for (int i = tid; i < P.hslots; i += NCT) { hkey[i] = kEmptySlot; hcnt[i] = 0u; }
    if (tid == 0) { ctl->status = 0; ctl->nuniq = 0u; }
    __syncthreads();
    const int64_t h0 = __ldg(P.hist_offsets + r), h1 = __ldg(P.hist_offsets + r + 1);
    uint32_t bad = 0;
    for (int64_t i = h0 + tid; i < h1; i += NCT) {
        const int64_t gid = __ldg(P.hist_ids + i);
        if (gid < 0 || gid >= P.vocab_total) { bad |= FG_ROW_BAD_HISTORY; continue; }
        const int64_t c = gid - P.vocab_offset;
        if (c < 0 || c >= P.vocab) continue;
        const uint32_t cc = (uint32_t)c;
        uint32_t h = col_hash(cc, mask);
        bool done = false;
        for (int probe = 0; probe <= (int)mask; ++probe) {
            const uint32_t k = atomicCAS(&hkey[h], kEmptySlot, cc);
            if (k == kEmptySlot) {
                const uint32_t pos = atomicAdd(&ctl->nuniq, 1u);   // first sighting: a new column
                if (pos < (uint32_t)P.hu_cap) srt[pos] = cc;
            }
            if (k == kEmptySlot || k == cc) { atomicAdd(&hcnt[h], 1u); done = true; break; }
            h = (h + 1u) & mask;
        }
        if (!done) bad |= FG_ROW_BAD_PARAM;   // more distinct ids than hist_max_len allows
    }
    if (bad) atomicOr(reinterpret_cast<unsigned int*>(&ctl->status), bad);
    __syncthreads();
    const uint32_t total = ctl->nuniq;
    const uint32_t U = min(total, (uint32_t)P.hu_cap);
    uint32_t* hc = g_hcol(P, r);
    uint32_t* hn = g_hcnt(P, r);
    for (uint32_t i = tid; i < U; i += NCT) {
        const uint32_t c = srt[i];
        uint32_t h = col_hash(c, mask), count = 0;
        for (int probe = 0; probe <= (int)mask; ++probe) {
            if (hkey[h] == c) { count = hcnt[h]; break; }
            h = (h + 1u) & mask;
        }
        hc[i] = c; hn[i] = count;
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t fl = (uint32_t)ctl->status;
        if (total > (uint32_t)P.hu_cap) fl |= FG_ROW_BAD_PARAM;
        hh->nh = U;
        hh->flags = fl;
    }
}

// ===========================================================================
// K2: the stream
// ===========================================================================
struct St {
    float mx;          // NaN-propagating maximum of the raw row
    float bv;          // greedy: best non-history value and its first column
    uint32_t bc;
    float zm, nzc;     // sum of exp: running reference and -(zm * c)
    float z0, z1;
    float c;           // log2(e) / T
    float tau;         // candidate filter (x >= tau)
    bool cand;         // the buffer is still complete above tau
};

__device__ __forceinline__ void append(const Params& P, const Sm& s, float x, uint32_t col) {
    const uint32_t pos = atomicAdd(&s.ctl->ncand, 1u);
    if (pos < (uint32_t)P.cap) { s.ckey[pos] = fkey(x); s.ccol[pos] = col; } else s.ctl->ovf = 1u;
}

__device__ __forceinline__ void zadd(St& st, float x) {
    if (x > st.zm) {
        const float nn = -(x * st.c);
        const float f = ex2f_approx(nn - st.nzc);
        st.z0 *= f; st.z1 *= f;
        st.zm = x; st.nzc = nn;
    }
    st.z0 += ex2f_approx(__fmaf_rn(x, st.c, st.nzc));
}

// One tile's chunks. CLS: RC_GREEDY, RC_TOPK or RC_NUCLEUS (also for
// RC_FULL). PEN: the row has history columns; a chunk's history elements are
// set to -inf (one bitmap word per chunk), so the maximum, the argmax, the
// candidates and the sum of exp cover the non-history columns only, and K3
// adds the history columns with their penalised values.
template <int DT, int CLS, bool PEN>
__device__ __forceinline__ void tile_chunks(const Params& P, const Sm& s, const uint4 (&v)[CPT], int nch, int tcol0,
                                            St& st) {
    constexpr int VEC = Elem<DT>::VEC;
    const int tid = threadIdx.x;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
        const int ch = tid + j * NCT;
        if (ch >= nch) continue;
        const int c0 = tcol0 + ch * VEC;
        uint4 x = v[j];
        if (PEN) {
            const uint32_t hb = hist_bits<VEC>(s.hbm, (uint32_t)c0);
            if (hb) {
#pragma unroll
                for (int e = 0; e < VEC; ++e)
                    if ((hb >> e) & 1u) elem_mask_inf<DT>(x, e);
            }
        }
        const float cm = chunk_max<DT>(x);
        st.mx = fmax_nan(st.mx, cm);
        if constexpr (CLS == RC_GREEDY) {
            if (cm > st.bv) {
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    const float xe = elem_at<DT>(x, e);
                    if (xe > st.bv) { st.bv = xe; st.bc = (uint32_t)(c0 + e); }
                }
            }
        } else {
            if constexpr (CLS == RC_NUCLEUS) {
                if (cm > st.zm) {
                    const float nn = -(cm * st.c);
                    const float f = ex2f_approx(nn - st.nzc);
                    st.z0 *= f; st.z1 *= f;
                    st.zm = cm; st.nzc = nn;
                }
#pragma unroll
                for (int e = 0; e < VEC; e += 2) {
                    st.z0 += ex2f_approx(__fmaf_rn(elem_at<DT>(x, e), st.c, st.nzc));
                    st.z1 += ex2f_approx(__fmaf_rn(elem_at<DT>(x, e + 1), st.c, st.nzc));
                }
            }
            if (cm >= st.tau) {
                // every element at or above tau: one atomic per chunk
                uint32_t msk = 0u;
#pragma unroll
                for (int e = 0; e < VEC; ++e) msk |= (elem_at<DT>(x, e) >= st.tau ? 1u : 0u) << e;
                uint32_t pos = atomicAdd(&s.ctl->ncand, (uint32_t)__popc(msk));
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    if (!((msk >> e) & 1u)) continue;
                    if (pos < (uint32_t)P.cap) {
                        s.ckey[pos] = fkey(elem_at<DT>(x, e));
                        s.ccol[pos] = (uint32_t)(c0 + e);
                    } else {
                        s.ctl->ovf = 1u;
                    }
                    ++pos;
                }
            }
        }
    }
}

// Starting threshold: a lower bound of the K0-th largest element of the first
// tile (K0 its share of the row's target, with a margin): histograms of the
// tile's chunk maxima give the lowest key of the bin that holds the K0-th
// largest maximum; at least K0 chunks, hence K0 elements, lie at or above it.
// -inf when the tile has fewer chunks. A guess for the row: the decision
// checks that the candidates hold the K-th largest.
template <int DT>
__device__ __noinline__ float tile0_tau(const Params& P, int kt, int nch, uint4 v0, uint4 v1, uint4 v2, uint4 v3) {
    static_assert(CPT == 4, "tile0_tau takes CPT chunks by value");
    constexpr int VEC = Elem<DT>::VEC;
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    const uint4 v[CPT] = {v0, v1, v2, v3};
    uint32_t km[CPT];
    uint32_t kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
        km[j] = 0u;
        if (tid + j * NCT >= nch) continue;
        const float cm = chunk_max<DT>(v[j]);
        if (!(cm == cm)) continue;
        km[j] = fkey(cm);
        kmin = min(kmin, km[j]); kmax = max(kmax, km[j]);
    }
    const int64_t share = ((int64_t)3 * kt * (int64_t)(nch * VEC) + 2 * P.vocab - 1) / (2 * P.vocab) + 8;
    const int K0 = (int)min((int64_t)nch, min((int64_t)kt, share));
    c_minmax_u32(kmin, kmax, s);
    if (kmin > kmax || K0 < 1) return -INFINITY;
    // two rounds of a 256-bin histogram: the whole key range, then the bin that
    // holds the K0-th largest maximum (a range that crosses zero or spans many
    // binades leaves the first round's bins too coarse)
    uint32_t lo = kmin, hi = kmax;
    uint64_t rank = (uint64_t)(K0 - 1);
    for (int round = 0; round < 2; ++round) {
        const int vb = varying_bits(0u, hi - lo);
        const int shift = vb > 8 ? vb - 8 : 0;
        for (int b = tid; b < NB; b += NCT) s.bcnt[b] = 0u;
        csync();
#pragma unroll
        for (int j = 0; j < CPT; ++j)
            if (km[j] != 0u && km[j] >= lo && km[j] <= hi) atomicAdd(&s.bcnt[(km[j] - lo) >> shift], 1u);
        csync();
        if (tid < 32) scan_desc<false>(s, NB, rank);
        csync();
        const SelRes rr = s.ctl->sel;
        csync();
        if (!rr.ok) return -INFINITY;
        const uint32_t blo = lo + (rr.key << shift);
        if (shift == 0) return funkey(blo);
        rank -= rr.before;
        hi = min(hi, blo + ((1u << shift) - 1u));
        lo = blo;
    }
    return funkey(lo);
}

// Compaction in one pass: a 256-bin histogram of the buffer's keys over their
// range; tau rises to the lowest key of the bin that holds the kt-th largest
// (so at least kt entries stay), closed under equal y. Returns the new count.
constexpr int CAP_MAX = 4096;
constexpr int PER_MAX = CAP_MAX / NCT;
__device__ __noinline__ uint32_t compact(const Params& P, int r, uint32_t n, int kt) {
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    const RowP p = load_row_params(P.temperature, P.top_p, P.top_k, P.rep, P.pres, P.freq, P.greedy, P.uniforms, r,
                                   false, P.vocab);
    if (n > (uint32_t)P.cap) n = (uint32_t)P.cap;
    if (n <= (uint32_t)kt) return n;
    uint32_t kmin = 0xffffffffu, kmax = 0u;
    for (uint32_t i = tid; i < n; i += NCT) { const uint32_t k = s.ckey[i]; kmin = min(kmin, k); kmax = max(kmax, k); }
    c_minmax_u32(kmin, kmax, s);
    const int vb = varying_bits(0u, kmax - kmin);
    const int shift = vb > 8 ? vb - 8 : 0;
    for (int b = tid; b < NB; b += NCT) s.bcnt[b] = 0u;
    csync();
    for (uint32_t i = tid; i < n; i += NCT) atomicAdd(&s.bcnt[(s.ckey[i] - kmin) >> shift], 1u);
    csync();
    if (tid < 32) scan_desc<false>(s, NB, (uint64_t)(kt - 1));
    csync();
    const SelRes rr = s.ctl->sel;
    csync();
    if (!rr.ok) return n;
    const uint32_t klow = kmin + (rr.key << shift);
    const float tnew = xmin_for_y(p, funkey(klow));
    if (tid == 0 && tnew > s.ctl->tau) s.ctl->tau = tnew;
    uint32_t kk[PER_MAX], ii[PER_MAX];
#pragma unroll
    for (int j = 0; j < PER_MAX; ++j) {
        const uint32_t idx = (uint32_t)(j * NCT + tid);
        kk[j] = idx < n ? s.ckey[idx] : 0u;
        ii[j] = idx < n ? s.ccol[idx] : 0u;
    }
    if (tid == 0) s.ctl->b32[0] = 0u;
    csync();   // every entry is in registers, tau is published
    const uint32_t kmin2 = fkey(s.ctl->tau);
    uint32_t cnt = 0;
#pragma unroll
    for (int j = 0; j < PER_MAX; ++j) cnt += ((uint32_t)(j * NCT + tid) < n && kk[j] >= kmin2) ? 1u : 0u;
    const int lane = tid & 31;
    const uint32_t incl = warp_incl_scan_u32(cnt, lane);
    uint32_t base = 0;
    if (lane == 31) base = atomicAdd(&s.ctl->b32[0], incl);
    base = __shfl_sync(0xffffffffu, base, 31) + incl - cnt;
#pragma unroll
    for (int j = 0; j < PER_MAX; ++j)
        if ((uint32_t)(j * NCT + tid) < n && kk[j] >= kmin2) { s.ckey[base] = kk[j]; s.ccol[base] = ii[j]; ++base; }
    csync();
    const uint32_t m = s.ctl->b32[0];
    csync();
    return m;
}

// A row K2 does not stream: top-k above the candidate limit (the cluster
// kernel samples it) and rows with invalid parameters.
__device__ __forceinline__ bool row_skipped(const Params& P, int r) {
    const float T = __ldg(P.temperature + r);
    const bool g = P.greedy ? (__ldg(P.greedy + r) != 0) : false;
    if (g || T == 0.0f) return false;
    const int tk = __ldg(P.top_k + r);
    const float tp = __ldg(P.top_p + r);
    const float u = __ldg(P.uniforms + r);
    if (!(T > 0.0f) || !(tp > 0.0f && tp <= 1.0f) || !(u >= 0.0f && u < 1.0f)) return true;
    return tk > P.k_fast && tk < P.vocab;
}
// Rows that sum exp over the whole row go first.
__device__ __forceinline__ bool row_heavy(const Params& P, int r) {
    const float T = __ldg(P.temperature + r);
    const bool g = P.greedy ? (__ldg(P.greedy + r) != 0) : false;
    if (g || T == 0.0f) return false;
    return __ldg(P.top_k + r) <= 0;
}

template <int DT>
__device__ void producer(const Params& P) {
    const Sm s = carve(P);
    const uint32_t ns = (uint32_t)P.nstage;
    const unsigned B = (unsigned)P.batch;
    volatile int* abort = &s.ctl->abort;
    uint32_t st = 0, ph = 0, k = 0;
    auto fetch = [&]() -> int {
        for (;;) {
            const unsigned v = atomicAdd(&P.ws[0], 1u);
            if (v >= 2u * B) return -1;
            const int r = (int)(v % B);
            if ((v < B) == row_heavy(P, r)) return r;
        }
    };
    int e = fetch();
    for (;;) {
        const uint32_t slot = k % RQ, rph = (k / RQ) & 1u;
        if (!mbar_wait(&s.rempty[slot], rph ^ 1u, abort)) { *abort = 1; return; }
        const bool skip = e >= 0 && row_skipped(P, e);
        s.ctl->rowq[slot] = e < 0 ? 0xffffffffu : ((uint32_t)e | (skip ? kSkip : 0u));
        mbar_arrive(&s.rfull[slot]);
        ++k;
        if (e < 0) return;
        if (!skip) {
            const Geom g = row_geom<Elem<DT>::SIZE>(P.logits, P.row_stride, P.vocab, e);
            const int nt = (int)((g.ibytes + TILE - 1) / TILE);
            for (int t = 0; t < nt; ++t) {
                if (!mbar_wait(&s.empty[st], ph ^ 1u, abort)) { *abort = 1; return; }
                const int64_t off = (int64_t)t * TILE;
                const int64_t left = g.ibytes - off;
                const uint32_t bytes = (uint32_t)(left < TILE ? left : TILE);
                mbar_arrive_expect_tx(&s.full[st], bytes);
                bulk_g2s(s.ring + (int64_t)st * TILE, g.interior + off, bytes, &s.full[st]);
                if (++st == ns) { st = 0; ph ^= 1u; }
            }
        }
        e = fetch();
    }
}

struct Ring { uint32_t st, ph; };

template <int DT, int CLS, bool PEN>
__device__ __noinline__ void stream_row(const Params& P, int r, Ring& rg, St& st_io, int kt) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE;
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const uint32_t ns = (uint32_t)P.nstage;
    const Geom g = row_geom<ESZ>(P.logits, P.row_stride, P.vocab, r);
    const int nt = (int)((g.ibytes + TILE - 1) / TILE);
    St st = st_io;
    volatile int* abort = &s.ctl->abort;
    // the buffer holds non-history columns only: compactions keep kt entries.
    // The count is checked after every second tile; a compaction starts while a
    // quarter of the buffer is still free, so two tiles rarely overflow it.
    const int kt2 = min(kt, P.cap / 2);
    uint32_t trig = (uint32_t)min(P.cap * 3 / 4, max(2 * kt2 + 256, 512));
    for (int t = 0; t < nt; ++t) {
        const bool ok = mbar_wait(&s.full[rg.st], rg.ph, abort);
        if (!ok) *abort = 1;
        const int64_t left = g.ibytes - (int64_t)t * TILE;
        const int nch = ok ? (int)((left < TILE ? left : TILE) / 16) : 0;
        const uint8_t* tile = s.ring + (int64_t)rg.st * TILE;
        uint4 v[CPT];
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            const int ch = tid + j * NCT;
            v[j] = ch < nch ? *reinterpret_cast<const uint4*>(tile + (int64_t)ch * 16) : make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[rg.st]);
        if (++rg.st == ns) { rg.st = 0; rg.ph ^= 1u; }
        const int tcol0 = g.head + t * (TILE / ESZ);
        if (CLS != RC_GREEDY && t == 0) st.tau = tile0_tau<DT>(P, kt, nch, v[0], v[1], v[2], v[3]);
        tile_chunks<DT, CLS, PEN>(P, s, v, nch, tcol0, st);
        if (CLS != RC_GREEDY) {
            if ((t & 1) || t == nt - 1) {
                csync();
                const uint32_t n = s.ctl->ncand;
                const bool ovf = s.ctl->ovf != 0u;
                csync();
                if (ovf) {
                    st.cand = false;
                } else if (st.cand && n > trig) {
                    if (tid == 0) s.ctl->tau = st.tau;   // the compaction only raises it
                    const uint32_t m = compact(P, r, n, kt2);
                    if (tid == 0) s.ctl->ncand = m;
                    st.tau = s.ctl->tau;
                    csync();
                    // ties may keep the count up: compact again only after 512 more
                    if (m + 512u > trig) trig = min((uint32_t)P.cap * 3 / 4, m + 512u);
                }
            }
        }
    }
    st_io = st;
}

template <int DT, int CLS, bool PEN>
__device__ __noinline__ void sample_row_cls(const Params& P, int r, Ring& rg) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE;
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    const RowP p = load_row_params(P.temperature, P.top_p, P.top_k, P.rep, P.pres, P.freq, P.greedy, P.uniforms, r,
                                   PEN, P.vocab);
    const Geom g = row_geom<ESZ>(P.logits, P.row_stride, P.vocab, r);
    const int kt = CLS == RC_TOPK ? p.K : P.k_nuc;
    St st;
    st.mx = -INFINITY; st.bv = -INFINITY; st.bc = 0xffffffffu;
    st.c = p.temp_on ? __fdiv_rn(kL2E, p.T) : kL2E;
    st.zm = -1e30f; st.nzc = -(st.zm * st.c); st.z0 = 0.0f; st.z1 = 0.0f;
    st.tau = -INFINITY; st.cand = true;
    stream_row<DT, CLS, PEN>(P, r, rg, st, kt);
    // the ragged head / tail (fewer than VEC each)
    {
        const int nh = g.head, ntl = P.vocab - g.tail0;
        if (tid < nh + ntl) {
            const int c = tid < nh ? tid : g.tail0 + (tid - nh);
            const float x = E::load(g.row, c);
            const bool hist = PEN && hist_bit(s.hbm, (uint32_t)c);
            if (!hist) {
                st.mx = fmax_nan(st.mx, x);
                if (CLS == RC_GREEDY) {
                    if (arg_better(x, (uint32_t)c, st.bv, st.bc)) { st.bv = x; st.bc = (uint32_t)c; }
                } else {
                    if (CLS == RC_NUCLEUS) zadd(st, x);
                    if (st.cand && x >= st.tau) append(P, s, x, (uint32_t)c);
                }
            }
        }
    }
    if (PEN) {
        // the history columns' raw values, right after the row streamed through
        // L2, penalised with K1's counts; their maximum and best entry
        const uint32_t U = min(hist_hdr(P, r)->nh, (uint32_t)P.hu_cap);
        const uint32_t* hc = g_hcol(P, r);
        const uint32_t* hn = g_hcnt(P, r);
        float* hp = g_hpen(P, r);
        float hm = -INFINITY, pb = -INFINITY;
        uint32_t pc = 0xffffffffu;
        for (uint32_t i = tid; i < U; i += NCT) {
            const uint32_t c = __ldcg(hc + i);
            const float pen = penalize(p, E::load(g.row, c), __ldcg(hn + i));
            hp[i] = pen;
            hm = fmax_nan(hm, pen);
            if (arg_better(pen, c, pb, pc)) { pb = pen; pc = c; }
        }
        hm = c_max_nan(hm, s);
        c_argmax(pb, pc, s);
        if (tid == 0) {
            HistHdr* hw = hist_hdr(P, r);
            hw->hmax = hm; hw->pbest = pb; hw->pcol = pc;
        }
    }
    csync();
    const bool ovf = s.ctl->ovf != 0u;
    const uint32_t n = min(s.ctl->ncand, (uint32_t)P.cap);
    const bool aborted = s.ctl->abort != 0;
    csync();
    const float M = c_max_nan(st.mx, s);
    if (CLS == RC_GREEDY) {
        float bv = st.bv;
        uint32_t bc = st.bc;
        c_argmax(bv, bc, s);
        if (tid == 0) {
            int status = p.bad | FG_ROW_GREEDY;
            int64_t out = -1;
            float Mf = M;   // the maximum after penalties
            if (PEN) {
                const HistHdr* hh = hist_hdr(P, r);
                status |= (int)hh->flags;
                Mf = fmax_nan(M, hh->hmax);
                if (arg_better(hh->pbest, hh->pcol, bv, bc)) { bv = hh->pbest; bc = hh->pcol; }
            }
            bool defer = false;
            if (aborted) status |= FG_ROW_TIMEOUT;
            else if (status & (FG_ROW_BAD_PARAM | FG_ROW_BAD_UNIFORM)) out = -1;
            else if (Mf != Mf) defer = true;          // the first NaN: the cluster kernel finds it
            else out = (Mf == -INFINITY) ? 0 : (int64_t)bc;
            if (defer) {
                P.out_ids[r] = kDeferredId;
            } else {
                P.out_ids[r] = out >= 0 ? out + P.vocab_offset : -1;
                if (P.out_status) P.out_status[r] = status;
            }
        }
    } else {
        // the candidates and statistics go to the row's block; K3 decides
        double zc = 0.0;
        if (CLS == RC_NUCLEUS && M == M && M > -INFINITY && M < INFINITY) {
            const double zs = (double)st.z0 + (double)st.z1;
            if (zs > 0.0) zc = zs * exp2(-(double)st.nzc - (double)M * (double)st.c);
        }
        if (CLS == RC_NUCLEUS) zc = c_sum_f64(zc, s);
        uint32_t* gk = g_ckey(P, r);
        uint32_t* gc = g_ccol(P, r);
        for (uint32_t i = tid; i < n; i += NCT) { gk[i] = s.ckey[i]; gc[i] = s.ccol[i]; }
        if (tid == 0) {
            RowStat* rs = row_stat(P, r);
            rs->zr = zc;
            rs->mraw = M;
            rs->tau = st.tau;
            rs->n = n;
            rs->ovf = (ovf || !st.cand || aborted) ? 1u : 0u;
            if (aborted) {
                P.out_ids[r] = -1;
                if (P.out_status) P.out_status[r] = FG_ROW_TIMEOUT;
            } else {
                P.out_ids[r] = kPendingId;
            }
        }
    }
    csync();
}

template <int DT>
__device__ void consumer(const Params& P) {
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    Ring rg{0u, 0u};
    if (P.pen_possible)
        for (int i = tid; i <= P.nwords; i += NCT) s.hbm[i] = 0u;   // ordered by the loop's first barrier
    volatile int* abort = &s.ctl->abort;
    for (uint32_t k = 0;; ++k) {
        const uint32_t slot = k % RQ, ph = (k / RQ) & 1u;
        if (tid == 0) {
            const bool ok = mbar_wait(&s.rfull[slot], ph, abort);
            s.ctl->snap = ok ? s.ctl->rowq[slot] : 0xfffffffeu;
            s.ctl->b32[3] = ok ? k + 1 : k;   // next slot to read after an abort
        }
        csync();
        const uint32_t q = s.ctl->snap;
        csync();
        if (q == 0xfffffffeu) break;                       // abort
        if (tid == 0) mbar_arrive(&s.rempty[slot]);
        if (q == 0xffffffffu) break;                       // no rows left
        const int r = (int)(q & ~kSkip);
        const bool has_hist = P.pen_possible && (__ldg(P.hist_offsets + r + 1) > __ldg(P.hist_offsets + r));
        const RowP p = load_row_params(P.temperature, P.top_p, P.top_k, P.rep, P.pres, P.freq, P.greedy, P.uniforms,
                                       r, has_hist, P.vocab);
        if (q & kSkip) {
            if (tid == 0) {
                if (p.bad) {
                    P.out_ids[r] = -1;
                    if (P.out_status) P.out_status[r] = p.bad;
                } else {
                    P.out_ids[r] = kDeferredId;
                }
            }
            continue;
        }
        if (tid == 0) { s.ctl->ncand = 0u; s.ctl->ovf = 0u; s.ctl->tau = -INFINITY; }
        uint32_t U = 0;
        const uint32_t* hc = nullptr;
        if (p.pen) {
            // the row's history columns from K1 into the (all-zero) bitmap: the
            // stream leaves them out, K3 adds their penalised values
            U = min(hist_hdr(P, r)->nh, (uint32_t)P.hu_cap);
            hc = g_hcol(P, r);
            for (uint32_t i = tid; i < U; i += NCT) {
                const uint32_t c = __ldcg(hc + i);
                atomicOr(&s.hbm[c >> 5], 1u << (c & 31u));
            }
        }
        csync();
        if (p.pen) {
            if (p.cls == RC_GREEDY) sample_row_cls<DT, RC_GREEDY, true>(P, r, rg);
            else if (p.cls == RC_TOPK) sample_row_cls<DT, RC_TOPK, true>(P, r, rg);
            else sample_row_cls<DT, RC_NUCLEUS, true>(P, r, rg);
            // sample_row_cls ends with a barrier: every lookup of this row is done
            for (uint32_t i = tid; i < U; i += NCT) s.hbm[__ldcg(hc + i) >> 5] = 0u;
        } else {
            if (p.cls == RC_GREEDY) sample_row_cls<DT, RC_GREEDY, false>(P, r, rg);
            else if (p.cls == RC_TOPK) sample_row_cls<DT, RC_TOPK, false>(P, r, rg);
            else sample_row_cls<DT, RC_NUCLEUS, false>(P, r, rg);
        }
        if (*abort) break;
    }
    if (tid == 0 && *abort) {
        // rows published to this CTA and not sampled, then every unclaimed
        // row, are reported as timed out (bounded waits: the producer has
        // stopped publishing)
        for (uint32_t k = s.ctl->b32[3];; ++k) {
            const uint32_t slot = k % RQ, ph = (k / RQ) & 1u;
            if (!mbar_wait_for(&s.rfull[slot], ph, 10000000ull)) break;
            const uint32_t q = s.ctl->rowq[slot];
            mbar_arrive(&s.rempty[slot]);
            if (q == 0xffffffffu) break;
            const int rr = (int)(q & ~kSkip);
            P.out_ids[rr] = -1;
            if (P.out_status) P.out_status[rr] = FG_ROW_TIMEOUT;
        }
        for (;;) {
            const unsigned v = atomicAdd(&P.ws[0], 1u);
            if (v >= 2u * (unsigned)P.batch) break;
            const int rr = (int)(v % (unsigned)P.batch);
            if ((v < (unsigned)P.batch) != row_heavy(P, rr)) continue;
            P.out_ids[rr] = -1;
            if (P.out_status) P.out_status[rr] = FG_ROW_TIMEOUT;
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(NTH, 2) stream_kernel(const __grid_constant__ Params P) {
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < P.nstage; ++i) { mbar_init(&s.full[i], 1); mbar_init(&s.empty[i], NCW); }
        for (int i = 0; i < RQ; ++i) { mbar_init(&s.rfull[i], 1); mbar_init(&s.rempty[i], 1); }
        s.ctl->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid >= NCT) {
        if (tid == NCT) producer<DT>(P);
        return;
    }
    consumer<DT>(P);
    csync();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(&P.ws[1], 1u) == gridDim.x - 1) {
            P.ws[0] = 0u;
            P.ws[1] = 0u;
            __threadfence();
        }
    }
}

// ---------------------------------------------------------------------------
// Finish of a row decided in the candidate buffer. Entries [0, n): x-keys
// and columns; the buffer holds every element with x >= tau. Returns false
// when the row cannot be decided there (the caller defers it).
// ---------------------------------------------------------------------------
struct Fin {
    int64_t id;
    int status;
    bool defer;
    bool deep;          // deferred because the cut or the draw lies below the candidates
    double zq;          // then: the row's total mass and the candidates' mass
    uint64_t ac;
};
__device__ __noinline__ Fin finish_sampling(const Params& P, int r, uint32_t n, float M, double Zd, float zmax) {
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    const bool has_hist = P.pen_possible && (__ldg(P.hist_offsets + r + 1) > __ldg(P.hist_offsets + r));
    const RowP p = load_row_params(P.temperature, P.top_p, P.top_k, P.rep, P.pres, P.freq, P.greedy, P.uniforms, r,
                                   has_hist, P.vocab);
    Fin fo;
    fo.id = -1; fo.status = 0; fo.defer = false; fo.deep = false; fo.zq = 0.0; fo.ac = 0;
    const float scale = __uint_as_float((uint32_t)(127 + P.mass_shift) << 23);
    const float My = ydiv(p, M);
    const uint32_t ktau = fkey(s.ctl->tau);
    if (n > (uint32_t)P.cap) n = (uint32_t)P.cap;
    // C: entries at or above tau, as y-keys; others get key 0 (never selected)
    uint32_t nabove = 0, ylo = 0xffffffffu, yhi = 0u;
    for (uint32_t i = tid; i < n; i += NCT) {
        const uint32_t k = s.ckey[i];
        uint32_t yk = 0u;
        if (k >= ktau) {
            yk = fkey(ydiv(p, funkey(k)));
            ++nabove;
            ylo = min(ylo, yk); yhi = max(yhi, yk);
        }
        s.ckey[i] = yk;
    }
    nabove = c_sum_u32(nabove, s);
    c_minmax_u32(ylo, yhi, s);
    auto qm = [&](uint32_t yk) -> uint64_t { return qmass(funkey(yk), My, scale); };
    // ---- top-k threshold ----
    uint32_t ykK = 1u;   // every valid entry (keys >= 1)
    if (p.cls == RC_TOPK) {
        if (nabove < (uint32_t)p.K) { fo.defer = true; return fo; }
        const Sel so = c_select<false>(s, [&](auto&& f) {
            for (uint32_t i0 = 0; i0 < n; i0 += NCT) {
                const uint32_t i = i0 + tid;
                const uint32_t yk = i < n ? s.ckey[i] : 0u;
                f(i < n && yk != 0u, yk, 1ull);
            }
        }, (uint64_t)(p.K - 1), ylo, yhi);
        if (!so.ok) { fo.defer = true; return fo; }
        ykK = so.key;
    }
    // ---- masses of the kept part of C ----
    uint64_t loc = 0;
    for (uint32_t i = tid; i < n; i += NCT) {
        const uint32_t yk = s.ckey[i];
        if (yk != 0u && yk >= ykK) loc += qm(yk);
    }
    const uint64_t AC = c_sum_u64(loc, s);
    auto kept = [&](uint32_t yk) { return yk != 0u && yk >= ykK; };
    const uint32_t klo = max(ylo, ykK);
    // ---- total mass and the cut ----
    uint64_t Qf = 0;
    bool cut = false;
    uint32_t tstar = 0u;
    uint64_t before_t = 0, qt = 0;
    if (p.cls == RC_TOPK) {
        if (p.use_p) {
            const uint64_t Pt = (uint64_t)floor((double)p.top_p * (double)AC);
            const Sel so = c_select<true>(s, [&](auto&& f) {
                for (uint32_t i0 = 0; i0 < n; i0 += NCT) {
                    const uint32_t i = i0 + tid;
                    const uint32_t yk = i < n ? s.ckey[i] : 0u;
                    const bool v = i < n && kept(yk);
                    f(v, yk, v ? qm(yk) : 0ull);
                }
            }, Pt, klo, yhi);
            if (!so.ok) { fo.defer = true; return fo; }
            cut = true; tstar = so.key; before_t = so.before;
            qt = so.nat ? so.at / so.nat : 0;
            uint64_t m = so.nat;
            if (qt > 0) { const uint64_t mm = (Pt - so.before) / qt + 1; if (mm < m) m = mm; }
            Qf = so.before + m * qt;
        } else {
            Qf = AC;
        }
    } else {
        // top-k off: the row's total mass from the online sum of exp
        const double Zq = Zd * exp((double)zmax / (double)p.T - (double)My) * (double)scale;
        if (p.use_p) {
            const uint64_t Pt = (uint64_t)floor((double)p.top_p * Zq);
            if (Pt >= AC) {   // the cut lies below the buffer
                fo.defer = true; fo.deep = true; fo.zq = Zq; fo.ac = AC;
                return fo;
            }
            const Sel so = c_select<true>(s, [&](auto&& f) {
                for (uint32_t i0 = 0; i0 < n; i0 += NCT) {
                    const uint32_t i = i0 + tid;
                    const uint32_t yk = i < n ? s.ckey[i] : 0u;
                    const bool v = i < n && kept(yk);
                    f(v, yk, v ? qm(yk) : 0ull);
                }
            }, Pt, klo, yhi);
            if (!so.ok) { fo.defer = true; return fo; }
            cut = true; tstar = so.key; before_t = so.before;
            qt = so.nat ? so.at / so.nat : 0;
            uint64_t m = so.nat;
            if (qt > 0) { const uint64_t mm = (Pt - so.before) / qt + 1; if (mm < m) m = mm; }
            Qf = so.before + m * qt;
        } else {
            Qf = (uint64_t)Zq;
            const uint64_t Dt0 = (uint64_t)floor((double)p.u * (double)Qf);
            if (Dt0 >= AC) {   // the draw lies below the buffer
                fo.defer = true; fo.deep = true; fo.zq = Zq; fo.ac = AC;
                return fo;
            }
        }
    }
    if (Qf == 0) { fo.defer = true; return fo; }
    // ---- the draw ----
    uint64_t Dt = (uint64_t)floor((double)p.u * (double)Qf);
    if (Dt >= Qf) Dt = Qf - 1;
    uint32_t dkey;
    uint64_t dj;
    if (cut && Dt >= before_t) {
        dkey = tstar;
        dj = qt ? (Dt - before_t) / qt : 0;
    } else {
        const uint32_t ts = cut ? tstar : 0u;
        const Sel so = c_select<true>(s, [&](auto&& f) {
            for (uint32_t i0 = 0; i0 < n; i0 += NCT) {
                const uint32_t i = i0 + tid;
                const uint32_t yk = i < n ? s.ckey[i] : 0u;
                const bool v = i < n && kept(yk) && (!cut || yk > ts);
                f(v, yk, v ? qm(yk) : 0ull);
            }
        }, Dt, klo, yhi);
        if (!so.ok) { fo.defer = true; return fo; }
        dkey = so.key;
        const uint64_t qd = so.nat ? so.at / so.nat : 0;
        dj = qd ? (Dt - so.before) / qd : 0;
    }
    // ---- dj-th column (ascending) among the entries at dkey: select on ~column ----
    uint32_t cmin = 0xffffffffu, cmax = 0u;
    for (uint32_t i = tid; i < n; i += NCT)
        if (s.ckey[i] == dkey) { const uint32_t kc = ~s.ccol[i]; cmin = min(cmin, kc); cmax = max(cmax, kc); }
    c_minmax_u32(cmin, cmax, s);
    // descending ~column = ascending column; dj-th from the smallest column is
    // (count - 1 - dj)-th ... counted from the largest ~column
    const Sel sc = c_select<false>(s, [&](auto&& f) {
        for (uint32_t i0 = 0; i0 < n; i0 += NCT) {
            const uint32_t i = i0 + tid;
            const bool v = i < n && s.ckey[i] == dkey;
            f(v, v ? ~s.ccol[i] : 0u, 1ull);
        }
    }, dj, cmin, cmax);
    if (!sc.ok) { fo.defer = true; return fo; }
    fo.id = (int64_t)(~sc.key);
    return fo;
}


// ===========================================================================
// K3: decide the rows K2 left (out_ids == kPendingId)
// ===========================================================================
template <int DT>
__global__ void __launch_bounds__(NCT, 5) decide_kernel(const __grid_constant__ Params P) {
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    for (int r = blockIdx.x; r < P.batch; r += gridDim.x) {
        if (__ldcg(P.out_ids + r) != kPendingId) continue;
        const bool has_hist = P.pen_possible && (__ldg(P.hist_offsets + r + 1) > __ldg(P.hist_offsets + r));
        const RowP p = load_row_params(P.temperature, P.top_p, P.top_k, P.rep, P.pres, P.freq, P.greedy, P.uniforms,
                                       r, has_hist, P.vocab);
        const RowStat rs = *row_stat(P, r);
        const float scale = __uint_as_float((uint32_t)(127 + P.mass_shift) << 23);
        (void)scale;
        int status = p.bad;
        uint32_t U = 0;
        // Mraw: the maximum of the non-history columns (K2); Mf: after penalties
        const float Mraw = rs.mraw;
        float Mf = Mraw;
        if (p.pen) {
            const HistHdr* hh = hist_hdr(P, r);
            status |= (int)hh->flags;
            U = min(hh->nh, (uint32_t)P.hu_cap);
            Mf = fmax_nan(Mraw, hh->hmax);
        }
        bool defer = rs.ovf != 0u, deep = false;
        int64_t out = -1;
        if (status & (FG_ROW_BAD_PARAM | FG_ROW_BAD_UNIFORM)) {
            defer = false;
        } else if (Mf != Mf) {
            status |= FG_ROW_NAN; defer = false;
        } else if (Mf == INFINITY) {
            status |= FG_ROW_POS_INF; defer = false;
        } else if (Mf == -INFINITY) {
            status |= FG_ROW_ALL_MASKED; defer = false;
        } else if (!defer) {
            // the decision set: the candidates (non-history, raw = final) and the
            // history entries at or above tau with their penalised values
            const float tau = rs.tau;
            uint32_t n = min(rs.n, (uint32_t)P.cap);
            const uint32_t* gk = g_ckey(P, r);
            const uint32_t* gc = g_ccol(P, r);
            // the candidates hold no history column (K2 leaves them out)
            for (uint32_t i = tid; i < n; i += NCT) { s.ckey[i] = gk[i]; s.ccol[i] = gc[i]; }
            if (tid == 0) { s.ctl->ncand = n; s.ctl->tau = tau; s.ctl->ovf = 0u; }
            csync();
            // history entries at or above tau join the set
            float hmax = -INFINITY;
            if (p.pen) {
                const uint32_t* hc = g_hcol(P, r);
                const float* hp = g_hpen(P, r);
                for (uint32_t i = tid; i < U; i += NCT) {
                    const float pen = hp[i];
                    hmax = fmax_nan(hmax, pen);
                    if (pen >= tau) append(P, s, pen, hc[i]);
                }
            }
            hmax = c_max_nan(hmax, s);
            csync();
            n = s.ctl->ncand;
            if (s.ctl->ovf || n > (uint32_t)P.cap) defer = true;
            csync();
            if (!defer) {
                // the row's maximum after penalties: every value at or above tau is
                // in the set, and the maximum of the non-history columns is one of
                // them unless the set is empty
                float cmax = -INFINITY;
                for (uint32_t i = tid; i < n; i += NCT) cmax = fmaxf(cmax, funkey(s.ckey[i]));
                cmax = c_max_nan(cmax, s);
                const float M = fmax_nan(cmax, hmax);
                if (n == 0 || !(M >= tau) || M == INFINITY || M != M) {
                    defer = true;
                } else {
                    double Zd = 0.0;
                    if (p.cls != RC_TOPK) {
                        // the non-history sum of exp (relative to Mraw) plus the
                        // history columns' penalised terms, relative to M
                        const double c = (double)(p.temp_on ? __fdiv_rn(kL2E, p.T) : kL2E);
                        double hz = 0.0;
                        if (p.pen) {
                            const float* hp = g_hpen(P, r);
                            for (uint32_t i = tid; i < U; i += NCT) hz += exp2(((double)hp[i] - (double)M) * c);
                        }
                        const double hz_t = c_sum_f64(hz, s);
                        const double zr = rs.zr;
                        Zd = hz_t + (zr > 0.0 ? zr * exp2(((double)Mraw - (double)M) * c) : 0.0);
                    }
                    if (!defer) {
                        const Fin fo = finish_sampling(P, r, n, M, Zd, M);
                        if (fo.defer) defer = true;
                        if (fo.deep && DT != FG_DTYPE_F32) {
                            // K4 continues below the candidates (16-bit logits)
                            deep = true;
                            if (tid == 0) {
                                RowStat* w = row_stat(P, r);
                                w->zq = fo.zq; w->ac = fo.ac; w->mfin = M;
                            }
                        }
                        else out = fo.id;
                    }
                }
            }
        }
        if (tid == 0) {
            if (defer) {
                P.out_ids[r] = deep ? kDeepId : kDeferredId;
            } else {
                P.out_ids[r] = out >= 0 ? out + P.vocab_offset : -1;
                if (out < 0 && !(status & FG_ROW_ERROR_MASK)) status |= FG_ROW_ALL_MASKED;
                if (P.out_status) P.out_status[r] = status;
            }
        }
        csync();
    }
}


// ===========================================================================
// K4: 16-bit rows whose top-p cut or draw lies below the candidates
// (out_ids == kDeepId). Below tau every non-history value is one of the
// 65536 16-bit values, and equal values have equal masses, so one counting
// pass over the row gives exact masses: count(key) * mass(value) for the
// NBIN keys right below tau. The history columns below tau join with their
// penalised values. A descending scan finds the element at which the
// cumulative mass reaches a target; a second pass finds the j-th column
// (ascending) of a value's elements. Rows outside this window, or with a tie
// between a history value and a 16-bit value at the decision, go to the
// cluster kernel.
// ===========================================================================
constexpr int NBIN = 16384;            // slots of the 16-bit keys counted below tau
constexpr int SLOTS = NBIN / NCT;      // keys per thread range of the scan (<= NCT)
static_assert(SLOTS <= NCT, "one key per thread inside a range");
constexpr int HL_MAX = 64;             // history entries whose value lies in one key's cell
constexpr int DCH = 8;                 // K4 column pass: 16-byte chunks a thread loads at a time (DCH * VEC <= 64)
constexpr int DCH1 = 4;                // K4 counting pass: chunks a thread loads at a time
constexpr int DNT = 1024;              // K4 threads (set-up, counting, masses); NCT of them do the rest
constexpr int kDeepStaticSmem = 4096;  // bound on K4's static shared memory (scan buffer, control)

__device__ __forceinline__ uint32_t key16_of_bits(uint32_t u) { return (u & 0x8000u) ? (~u & 0xffffu) : (u | 0x8000u); }
__device__ __forceinline__ uint32_t bits_of_key16(uint32_t k) { return (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu); }
template <int DT>
__device__ __forceinline__ float val16(uint32_t k) {
    const uint32_t b = bits_of_key16(k);
    if constexpr (DT == FG_DTYPE_BF16) return __uint_as_float(b << 16);
    else return __half2float(__ushort_as_half((unsigned short)b));
}
// Largest key whose value is <= x (strict: < x).
template <int DT, bool STRICT>
__device__ __forceinline__ int key16_floor(float x) {
    uint32_t b;
    if constexpr (DT == FG_DTYPE_BF16) b = __bfloat16_as_ushort(__float2bfloat16_rd(x));
    else b = __half_as_ushort(__float2half_rd(x));
    int k = (int)key16_of_bits(b);
    while (k >= 0 && (STRICT ? !(val16<DT>((uint32_t)k) < x) : !(val16<DT>((uint32_t)k) <= x))) --k;
    return k;
}

// Slots of the 16-bit keys. For bf16 the 24832 keys of the values with
// |x| < 2^-30 (both signs, zero included) share one slot, the zone: their
// masses are equal in fp32 (e^(y - My) with |y| < 2^-29 / T), so slot sums
// stay exact, and a target that falls inside the zone hands the row on.
// NBIN slots below a tau of a few units then reach the most negative values.
template <int DT>
struct VK {
    static constexpr bool Z = DT == FG_DTYPE_BF16;
    static constexpr uint32_t ZLO = 0x4F7Fu;   // key of -2^-30
    static constexpr uint32_t ZHI = 0xB080u;   // key of +2^-30
    static constexpr uint32_t ZW = ZHI - ZLO - 1u;
    __device__ static uint32_t of(uint32_t k) { return !Z ? k : (k >= ZHI ? k - ZW + 1u : (k > ZLO ? ZLO + 1u : k)); }
    __device__ static bool zone(uint32_t vk) { return Z && vk == ZLO + 1u; }
    // a key of the slot (for the zone: one of its keys, whose mass all of them share)
    __device__ static uint32_t key(uint32_t vk) { return !Z ? vk : (vk > ZLO + 1u ? vk + ZW - 1u : vk); }
};

struct DeepCtl {
    int flag;                 // 1: the row goes to the cluster kernel
    int found;                // the scan found its unit / the column pass its column
    int ut;                   // unit: 0 = a 16-bit value (slot), 1 = a history entry
    int slot;                 // unit slot (key - klo)
    uint32_t col;             // history entry column / found column
    uint32_t nh;              // history entries gathered for the walk
    uint32_t nat;             // elements of the unit
    uint32_t owner;           // thread whose keys hold the target
    unsigned long long before, q, base;
    unsigned long long rem;   // the target's remainder inside the found key's cell
};
struct HEnt { float v; uint32_t c; };

// Exclusive scan of v over the consumer threads in descending thread order
// (thread NCT-1 first); returns the exclusive prefix, *total the sum.
__device__ __forceinline__ unsigned long long c_scan_desc_u64(unsigned long long v, const Sm& s, unsigned long long* total) {
    const int q = NCT - 1 - (int)threadIdx.x;          // position in the descending order
    __shared__ unsigned long long xch[NCT];
    xch[q] = v;
    csync();
    const unsigned long long w = xch[threadIdx.x];     // the value at position threadIdx.x
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const unsigned long long incl = warp_incl_scan_u64(w, lane);
    if (lane == 31) s.ctl->red64[wid] = incl;
    csync();
    unsigned long long off = 0, tot = 0;
#pragma unroll
    for (int i = 0; i < NCW; ++i) { const unsigned long long t = s.ctl->red64[i]; if (i < wid) off += t; tot += t; }
    xch[threadIdx.x] = off + incl - w;                 // exclusive prefix of position threadIdx.x
    csync();
    const unsigned long long ex = xch[q];
    csync();
    *total = tot;
    return ex;
}

// Draw among the candidates (all of them kept: the cut lies below them) with
// target Dt: the candidates' y-keys are in s.ckey (0: not a candidate).
__device__ __noinline__ int64_t cand_draw(const Sm& s, uint32_t n, float My, float scale, uint64_t Dt, uint32_t ylo,
                                          uint32_t yhi) {
    const int tid = threadIdx.x;
    auto qm = [&](uint32_t yk) -> uint64_t { return qmass(funkey(yk), My, scale); };
    const Sel so = c_select<true>(s, [&](auto&& f) {
        for (uint32_t i0 = 0; i0 < n; i0 += NCT) {
            const uint32_t i = i0 + tid;
            const uint32_t yk = i < n ? s.ckey[i] : 0u;
            const bool v = i < n && yk != 0u;
            f(v, yk, v ? qm(yk) : 0ull);
        }
    }, Dt, ylo, yhi);
    if (!so.ok) return -1;
    const uint32_t dkey = so.key;
    const uint64_t qd = so.nat ? so.at / so.nat : 0;
    const uint64_t dj = qd ? (Dt - so.before) / qd : 0;
    uint32_t cmin = 0xffffffffu, cmax = 0u;
    for (uint32_t i = tid; i < n; i += NCT)
        if (s.ckey[i] == dkey) { const uint32_t kc = ~s.ccol[i]; cmin = min(cmin, kc); cmax = max(cmax, kc); }
    c_minmax_u32(cmin, cmax, s);
    const Sel sc = c_select<false>(s, [&](auto&& f) {
        for (uint32_t i0 = 0; i0 < n; i0 += NCT) {
            const uint32_t i = i0 + tid;
            const bool v = i < n && s.ckey[i] == dkey;
            f(v, v ? ~s.ccol[i] : 0u, 1ull);
        }
    }, dj, cmin, cmax);
    if (!sc.ok) return -1;
    return (int64_t)(~sc.key);
}

template <int DT>
__global__ void __launch_bounds__(DNT, 1) deep_kernel(const __grid_constant__ Params P) {
    using E = Elem<DT>;
    constexpr int VEC = E::VEC;
    const Sm s = carve(P);
    const int tid = threadIdx.x;
    uint32_t* cnt = reinterpret_cast<uint32_t*>(ssmem + P.off_cnt);
    unsigned long long* tsum = reinterpret_cast<unsigned long long*>(ssmem + P.off_tsum);
    unsigned long long* hmass = tsum + NCT;   // SLOTS entries after the NCT range sums
    HEnt* hl = reinterpret_cast<HEnt*>(ssmem + P.off_hl);
    __shared__ DeepCtl dc;
    for (int r = blockIdx.x; r < P.batch; r += gridDim.x) {
        if (__ldcg(P.out_ids + r) != kDeepId) continue;
        const bool has_hist = P.pen_possible && (__ldg(P.hist_offsets + r + 1) > __ldg(P.hist_offsets + r));
        const RowP p = load_row_params(P.temperature, P.top_p, P.top_k, P.rep, P.pres, P.freq, P.greedy, P.uniforms,
                                       r, has_hist, P.vocab);
        const RowStat rs = *row_stat(P, r);
        const float scale = __uint_as_float((uint32_t)(127 + P.mass_shift) << 23);
        const float M = rs.mfin, My = ydiv(p, M);
        const float tau = rs.tau;
        const uint64_t AC = rs.ac;
        int status = p.bad;
        uint32_t U = 0;
        const uint32_t* hc = nullptr;
        const float* hp = nullptr;
        if (p.pen) {
            const HistHdr* hh = hist_hdr(P, r);
            status |= (int)hh->flags;
            U = min(hh->nh, (uint32_t)P.hu_cap);
            hc = g_hcol(P, r);
            hp = g_hpen(P, r);
        }
        const Geom g = row_geom<E::SIZE>(P.logits, P.row_stride, P.vocab, r);
        const int ktop_raw = key16_floor<DT, true>(tau);   // largest key below tau
        const int ktop = ktop_raw < 0 ? -1 : (int)VK<DT>::of((uint32_t)ktop_raw);   // its slot
        const int klo = ktop - (NBIN - 1);              // may be negative: those bins stay empty
        // ---- bitmap of the history columns; counters cleared ----
        // (set-up, counting and masses use all DNT threads; the scans and the
        // draw the first NCT, on the consumer-group barrier)
        if (P.pen_possible)
            for (int i = tid; i <= P.nwords; i += DNT) s.hbm[i] = 0u;
        for (int i = tid; i < NBIN; i += DNT) cnt[i] = 0u;
        if (tid == 0) { dc.flag = ktop < 0 ? 1 : 0; dc.found = 0; dc.nh = 0u; s.ctl->ovf = 0u; }
        __syncthreads();
        for (uint32_t i = tid; i < U; i += DNT) {
            const uint32_t c = __ldcg(hc + i);
            atomicOr(&s.hbm[c >> 5], 1u << (c & 31u));
        }
        __syncthreads();
        // ---- pass 1: counts of the non-history 16-bit values below tau ----
        auto count_elem = [&](uint32_t bits16) {
            // below tau iff the key is (keys are order-preserving)
            const int key = (int)key16_of_bits(bits16);
            if (key > ktop_raw) return;
            const int k = (int)VK<DT>::of((uint32_t)key) - klo;
            if (k >= 0) atomicAdd(&cnt[k], 1u);
        };
        const int64_t nchunks = g.ibytes / 16;
        const uint4* gin = reinterpret_cast<const uint4*>(g.interior);
        for (int64_t base = 0; base < nchunks; base += DCH1 * DNT) {
            uint4 v[DCH1];
#pragma unroll
            for (int j = 0; j < DCH1; ++j) {   // every load in flight before the counting
                const int64_t ch = base + j * DNT + tid;
                v[j] = ch < nchunks ? __ldg(gin + ch) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int j = 0; j < DCH1; ++j) {
                const int64_t ch = base + j * DNT + tid;
                if (ch >= nchunks) continue;
                const int c0 = g.head + (int)ch * VEC;
                const uint32_t hb = p.pen ? hist_bits<VEC>(s.hbm, (uint32_t)c0) : 0u;
                const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    if ((hb >> e) & 1u) continue;
                    count_elem((w[e >> 1] >> (16 * (e & 1))) & 0xffffu);
                }
            }
        }
        {
            const int nh = g.head, ntl = P.vocab - g.tail0;
            for (int i = tid; i < nh + ntl; i += DNT) {
                const int c = i < nh ? i : g.tail0 + (i - nh);
                if (p.pen && hist_bit(s.hbm, (uint32_t)c)) continue;
                count_elem(reinterpret_cast<const uint16_t*>(g.row)[c]);
            }
        }
        __syncthreads();
        // ---- masses per thread's keys (descending order: thread NCT-1 holds the largest) ----
        // the mass of each range of SLOTS keys: one warp per range, its lanes
        // over the range's keys, a shuffle reduction (no atomics)
        {
            const int lane = tid & 31;
            for (int rg = tid >> 5; rg < NCT; rg += DNT / 32) {
                unsigned long long m = 0;
                for (int k = rg * SLOTS + lane; k < (rg + 1) * SLOTS; k += 32) {
                    const uint32_t c = cnt[k];
                    if (c) m += (unsigned long long)c * qmass(ydiv(p, val16<DT>(VK<DT>::key((uint32_t)(k + klo)))), My, scale);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m += __shfl_xor_sync(0xffffffffu, m, o);
                if (lane == 0) tsum[rg] = m;
            }
        }
        __syncthreads();
        if (tid < NCT) {   // the rest of the row runs on the first NCT threads
        // history entries below tau, each with its own mass, at the key just below or at its value
        for (uint32_t i = tid; i < U; i += NCT) {
            const float v = hp[i];
            if (!(v < tau)) continue;
            const int k = (int)VK<DT>::of((uint32_t)key16_floor<DT, false>(v)) - klo;
            if (k < 0) continue;   // below the window
            atomicAdd(&tsum[k / SLOTS], qmass(ydiv(p, v), My, scale));
        }
        csync();
        // ---- find: the unit at which the cumulative mass below tau passes `target` ----
        // returns false (and flags the row) when it lies below the window
        auto find = [&](uint64_t target) -> bool {
            unsigned long long total = 0;
            const unsigned long long ex = c_scan_desc_u64(tsum[tid], s, &total);
            if (tid == 0) { dc.found = 0; dc.nh = 0u; }
            csync();
            if (target < total && ex <= target && target < ex + tsum[tid]) { dc.owner = (uint32_t)tid; dc.base = ex; }
            csync();
            if (!(target < total)) { if (tid == 0) dc.flag = 1; csync(); return false; }
            const int own = (int)dc.owner;
            const int k0 = own * SLOTS;
            // per key of the owner's range: the history entries in its cell [value(k), value(k+1))
            for (int j = tid; j < SLOTS; j += NCT) { hmass[j] = 0ull; }
            csync();
            for (uint32_t i = tid; i < U; i += NCT) {
                const float v = hp[i];
                if (!(v < tau)) continue;
                const int k = (int)VK<DT>::of((uint32_t)key16_floor<DT, false>(v)) - klo;
                if (k < k0 || k >= k0 + SLOTS) continue;
                atomicAdd(&hmass[k - k0], qmass(ydiv(p, v), My, scale));
            }
            csync();
            // one key per thread, threads NCT-SLOTS.. NCT-1 in ascending key order, so the
            // descending scan visits the keys from the largest down
            const int j = tid - (NCT - SLOTS);
            unsigned long long mk = 0;
            uint64_t qk = 0;
            if (j >= 0) {
                const uint32_t c = cnt[k0 + j];
                if (c) qk = qmass(ydiv(p, val16<DT>(VK<DT>::key((uint32_t)(k0 + j + klo)))), My, scale);
                mk = hmass[j] + (unsigned long long)c * qk;
            }
            unsigned long long tot2 = 0;
            const unsigned long long ex2 = c_scan_desc_u64(mk, s, &tot2);
            const uint64_t rem = target - dc.base;   // dc.base is not written in this step
            if (j >= 0 && ex2 <= rem && rem < ex2 + mk) {
                dc.slot = k0 + j;
                dc.before = AC + dc.base + ex2;   // mass before the key's cell
                dc.rem = rem - ex2;
            }
            csync();
            const int ks = dc.slot;
            // the cell's history entries (largest first), then the key's own elements
            for (uint32_t i = tid; i < U; i += NCT) {
                const float v = hp[i];
                if (!(v < tau)) continue;
                if ((int)VK<DT>::of((uint32_t)key16_floor<DT, false>(v)) - klo != ks) continue;
                const uint32_t pos = atomicAdd(&dc.nh, 1u);
                if (pos < (uint32_t)HL_MAX) { hl[pos].v = v; hl[pos].c = __ldcg(hc + i); }
            }
            csync();
            if (tid == 0) {
                const uint32_t nh = dc.nh;
                if (nh > (uint32_t)HL_MAX || VK<DT>::zone((uint32_t)(ks + klo))) {
                    dc.flag = 1;   // too many entries in the cell, or the target inside the zone
                } else {
                    // descending value, ascending column
                    for (uint32_t a = 1; a < nh; ++a) {
                        const HEnt x = hl[a];
                        uint32_t b = a;
                        while (b > 0 && (hl[b - 1].v < x.v || (hl[b - 1].v == x.v && hl[b - 1].c > x.c))) { hl[b] = hl[b - 1]; --b; }
                        hl[b] = x;
                    }
                    const float gy = ydiv(p, val16<DT>(VK<DT>::key((uint32_t)(ks + klo))));
                    const uint32_t c = cnt[ks];
                    uint64_t r2 = dc.rem, before = dc.before;
                    bool done = false;
                    for (uint32_t h = 0; h < nh && !done; ++h) {
                        const float hy = ydiv(p, hl[h].v);
                        if (hy == gy && c != 0u) { dc.flag = 1; done = true; break; }   // a tie across kinds
                        const uint64_t qh = qmass(hy, My, scale);
                        if (r2 < qh) {
                            dc.ut = 1; dc.col = hl[h].c; dc.nat = 1; dc.q = qh; dc.before = before;
                            dc.found = 1; done = true;
                        } else {
                            r2 -= qh; before += qh;
                        }
                    }
                    if (!done) {
                        const uint64_t q = qmass(gy, My, scale);
                        if (c == 0u || r2 >= (uint64_t)c * q) {
                            dc.flag = 1;   // rounding put the target past the cell: leave the row
                        } else if ((ks + klo < ktop && ydiv(p, val16<DT>(VK<DT>::key((uint32_t)(ks + klo + 1)))) == gy) ||
                                   (ks + klo > 0 && ydiv(p, val16<DT>(VK<DT>::key((uint32_t)(ks + klo - 1)))) == gy)) {
                            dc.flag = 1;   // equal y on a neighbouring 16-bit value would interleave columns
                        } else {
                            dc.ut = 0; dc.nat = c; dc.q = q; dc.before = before; dc.found = 1;
                        }
                    }
                }
            }
            csync();
            return dc.flag == 0 && dc.found != 0;
        };
        // ---- the j-th (ascending) non-history column with key (slot + klo) ----
        auto column = [&](int slot, uint64_t j) -> int64_t {
            const uint32_t kk = VK<DT>::key((uint32_t)(slot + klo));   // never the zone (it defers)
            if (tid == 0) { dc.found = 0; dc.base = 0; }
            csync();
            auto match = [&](int c, uint32_t bits16) {
                return key16_of_bits(bits16) == kk && !(p.pen && hist_bit(s.hbm, (uint32_t)c));
            };
            // ragged head first (thread 0), then the interior a tile of NCT chunks at a time, then the tail
            if (tid == 0) {
                uint64_t run = 0;
                for (int c = 0; c < g.head; ++c)
                    if (match(c, reinterpret_cast<const uint16_t*>(g.row)[c])) {
                        if (run == j) { dc.found = 1; dc.col = (uint32_t)c; break; }
                        ++run;
                    }
                dc.base = run;
            }
            csync();
            for (int64_t t0 = 0; t0 < nchunks && !dc.found; t0 += DCH * NCT) {
                // thread tid holds the DCH consecutive chunks from ch0: a scan in
                // thread order is a scan in column order
                const int64_t ch0 = t0 + (int64_t)tid * DCH;
                uint4 v[DCH];
#pragma unroll
                for (int q = 0; q < DCH; ++q)
                    v[q] = ch0 + q < nchunks ? __ldg(gin + ch0 + q) : make_uint4(0u, 0u, 0u, 0u);
                uint32_t m = 0u;
                unsigned long long mm = 0ull;   // matches; bit q*VEC+e of mm (DCH * VEC <= 64)
#pragma unroll
                for (int q = 0; q < DCH; ++q) {
                    if (ch0 + q >= nchunks) continue;
                    const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
                    const int c0 = g.head + (int)(ch0 + q) * VEC;
#pragma unroll
                    for (int e = 0; e < VEC; ++e)
                        if (match(c0 + e, (w[e >> 1] >> (16 * (e & 1))) & 0xffffu)) { mm |= 1ull << (q * VEC + e); ++m; }
                }
                // exclusive scan of m in thread order
                const int lane = tid & 31, wid = tid >> 5;
                const uint32_t incl = warp_incl_scan_u32(m, lane);
                if (lane == 31) s.ctl->red32[wid] = incl;
                csync();
                uint32_t off = 0, tot = 0;
#pragma unroll
                for (int i = 0; i < NCW; ++i) { const uint32_t t = s.ctl->red32[i]; if (i < wid) off += t; tot += t; }
                const uint64_t b0 = dc.base + off + incl - m;
                if (m && b0 <= j && j < b0 + m) {
                    uint32_t left = (uint32_t)(j - b0);
                    unsigned long long bits = mm;
                    while (left--) bits &= bits - 1ull;
                    dc.col = (uint32_t)(g.head + (int)ch0 * VEC + (__ffsll((long long)bits) - 1));
                    dc.found = 1;
                }
                csync();
                if (tid == 0) dc.base += tot;
                csync();
            }
            if (tid == 0 && !dc.found) {
                uint64_t run = dc.base;
                for (int c = g.tail0; c < P.vocab; ++c)
                    if (match(c, reinterpret_cast<const uint16_t*>(g.row)[c])) {
                        if (run == j) { dc.found = 1; dc.col = (uint32_t)c; break; }
                        ++run;
                    }
            }
            csync();
            const int64_t res = dc.found ? (int64_t)dc.col : -1;
            csync();
            return res;
        };
        // ---- the cut, then the draw ----
        int64_t out = -1;
        bool defer = dc.flag != 0;
        const double Zq = rs.zq;
        uint64_t Qf = 0, before_t = 0, qt = 0;
        int cut_ut = -1, cut_slot = 0;
        uint32_t cut_col = 0;
        bool cut = false;
        if (!defer && p.use_p) {
            const uint64_t Pt = (uint64_t)floor((double)p.top_p * Zq);
            if (Pt < AC || !find(Pt - AC)) {
                defer = true;
            } else {
                cut = true; cut_ut = dc.ut; cut_slot = dc.slot; cut_col = dc.col;
                before_t = dc.before; qt = dc.q;
                uint64_t m = dc.nat;
                if (qt > 0) { const uint64_t mm = (Pt - before_t) / qt + 1; if (mm < m) m = mm; }
                Qf = before_t + m * qt;
            }
        } else if (!defer) {
            Qf = (uint64_t)Zq;
        }
        if (!defer && Qf == 0) defer = true;
        if (!defer) {
            uint64_t Dt = (uint64_t)floor((double)p.u * (double)Qf);
            if (Dt >= Qf) Dt = Qf - 1;
            if (cut && Dt >= before_t) {
                const uint64_t dj = qt ? (Dt - before_t) / qt : 0;
                out = cut_ut == 1 ? (int64_t)cut_col : column(cut_slot, dj);
            } else if (Dt < AC) {
                // among the candidates: their y-keys, then the select
                const uint32_t n = min(rs.n, (uint32_t)P.cap);
                const uint32_t* gk = g_ckey(P, r);
                const uint32_t* gc = g_ccol(P, r);
                const uint32_t ktau = fkey(tau);
                uint32_t ylo = 0xffffffffu, yhi = 0u;
                for (uint32_t i = tid; i < n; i += NCT) {
                    const uint32_t k = gk[i];
                    uint32_t yk = 0u;
                    if (k >= ktau) { yk = fkey(ydiv(p, funkey(k))); ylo = min(ylo, yk); yhi = max(yhi, yk); }
                    s.ckey[i] = yk; s.ccol[i] = gc[i];
                }
                uint32_t nn = n;
                // the history entries at or above tau are candidates too
                if (p.pen) {
                    if (tid == 0) s.ctl->ncand = n;
                    csync();
                    for (uint32_t i = tid; i < U; i += NCT) {
                        const float v = hp[i];
                        if (!(v >= tau)) continue;
                        const uint32_t pos = atomicAdd(&s.ctl->ncand, 1u);
                        if (pos < (uint32_t)P.cap) {
                            const uint32_t yk = fkey(ydiv(p, v));
                            s.ckey[pos] = yk; s.ccol[pos] = __ldcg(hc + i);
                            ylo = min(ylo, yk); yhi = max(yhi, yk);
                        } else {
                            s.ctl->ovf = 1u;
                        }
                    }
                    csync();
                    nn = min(s.ctl->ncand, (uint32_t)P.cap);
                    if (s.ctl->ovf) defer = true;
                    csync();
                }
                c_minmax_u32(ylo, yhi, s);
                if (!defer) {
                    out = cand_draw(s, nn, My, scale, Dt, ylo, yhi);
                    if (out < 0) defer = true;
                }
            } else if (find(Dt - AC)) {
                const uint64_t dj = dc.q ? (Dt - dc.before) / dc.q : 0;
                out = dc.ut == 1 ? (int64_t)dc.col : column(dc.slot, dj);
            } else {
                defer = true;
            }
            if (out < 0) defer = true;
        }
        if (tid == 0) {
            if (defer) {
                P.out_ids[r] = kDeferredId;
            } else {
                P.out_ids[r] = out + P.vocab_offset;
                if (P.out_status) P.out_status[r] = status;
            }
        }
        csync();
        }
        __syncthreads();   // every thread, before the next row reuses shared memory
    }
}

}  // namespace strm
}  // namespace fg
