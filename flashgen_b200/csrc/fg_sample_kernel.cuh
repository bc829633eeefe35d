// fg_sample_kernel.cuh — layout, per-row parameters and block-level primitives
// of the fused decode-step sampler (sm_100a).
//
// Kernel structure (fg_kernels.cuh):
//   one persistent CTA per SM, rows handed out dynamically (global counter in
//   the caller's workspace) by a producer warp that also streams each row's
//   16-byte-aligned interior HBM -> shared memory with 1-D bulk async copies
//   (cp.async.bulk, completion counted on mbarriers) into a ring of 16 KB tiles;
//   NCW consumer warps per tile: history columns are masked out (their raw
//   values captured for a later merge), packed NaN-propagating max over whole
//   16-byte chunks, online sum-exp for rows whose top-p runs over the whole
//   vocabulary, and a candidate filter x >= xmin that appends (key, column)
//   pairs to a shared buffer; xmin is an exact lower bound of the K-th largest
//   value, raised by compactions (block radix select) when the buffer fills.
//   The epilogue decides the row on the candidates with integer (fixed-point)
//   masses; rows the candidates cannot decide use histogram passes over the
//   row re-read from L2.
//
// Reference semantics (FlashGen): flashgen/sampling/sampler.py:57-169,
// csrc/runtime/pipeline.cpp:267-342.
#pragma once

#include "fg_common.cuh"

namespace fg {

constexpr int NCW = 8;                  // consumer warps
constexpr int NCT = NCW * 32;           // consumer threads
constexpr int NTHREADS = NCT + 32;      // + one producer warp
constexpr int TILE_BYTES = 8192;        // one ring stage
constexpr int CPT = TILE_BYTES / 16 / NCT;  // 16-byte chunks per consumer thread per tile (2)
constexpr int CAND_CAP = 4096;          // candidate buffer entries
constexpr int HWM = 3072;               // compaction trigger (candidates after a check)
constexpr int K_FAST_MAX = 1536;        // largest top_k decided on the candidates
constexpr int K_NUCLEUS = 1536;         // candidate target for top-p-only / unfiltered rows
constexpr int NB = 256;                 // histogram bins (8-bit digits); NB == NCT
constexpr int RQ = 4;                   // row-queue slots
constexpr int BAR_CONS = 1;             // named barrier of the consumer warps

enum Mode : int { MODE_GREEDY = 0, MODE_TOPK = 1, MODE_NUCLEUS = 2, MODE_FULL = 3 };

// Per-call workspace (caller-owned, zero before the first call; every launch
// leaves it zero again).
struct Workspace {
    unsigned int next_row;
    unsigned int done_ctas;
    unsigned int pad[62];
};

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
    Workspace* ws;
    // candidates mode (vocabulary shards): per row, up to cand_max (y, global id)
    float* cand_vals;
    int32_t* cand_ids;
    int32_t* cand_count;
    int32_t cand_max;
    // shared-memory layout (byte offsets into dynamic smem)
    int32_t nstage;
    int32_t nwords;          // history bitmap words
    int32_t hu_cap;          // unique-history capacity (0: no penalties possible)
    int32_t off_ctl;         // RowCtl
    int32_t off_bins, off_cnts, off_ckey, off_cid;
    int32_t off_bitmap, off_prefix, off_counts, off_sval, off_scol, off_ring;
    int32_t pen_possible;
    int32_t mass_shift;      // S: masses are round(e * 2^S)
    int32_t id_bits;         // bits needed for a column index
    // ---- shard / merge / fixup stages of an earlier small-batch path (no
    //      entry point launches them: zero / null in every KParams built by
    //      fg_abi.cu): each row's columns cut into nshard shards sampled by
    //      different CTAs, whose candidates are merged
    // shard stage (nshard > 1): launch row r is shard r % nshard of row
    // r / nshard, columns [(r % nshard) * vocab, ... + vocab); candidates mode
    // with the outputs below, sorted by column
    int32_t nshard;
    double* cand_mz;           // [rows][2]: y maximum and sum of exp(y - that maximum)
    uint32_t* cand_thr;        // [rows]: y-key from which the row's output is complete
    // merge stage (merge_g > 0): launch row r is the union of row r's
    // merge_g shard outputs, already penalised and divided by T
    int32_t merge_g;
    const int32_t* id_map;     // [rows][vocab] global id of each union column
    const double* shard_mz;    // [rows * merge_g][2]
    const uint32_t* shard_thr; // [rows * merge_g]
    const int32_t* shard_status;
    int32_t* final_status;     // the caller's status array (rows finished here)
    // fixup stage (redo != null): only rows whose redo word has FG_ROW_SPLIT_REDO
    const int32_t* redo;
};

// Internal row status bit of the split path: the merge could not decide the
// row exactly from the shards' candidates; the fixup stage samples it whole.
constexpr int FG_ROW_SPLIT_REDO = 0x4000;

struct SelSlot {
    int ok;
    uint32_t digit, nat;
    uint64_t before, at;
};

struct RowCtl {
    int rowq[RQ];
    int abort;
    int status;
    int ovf[3];              // per-window overflow flags
    uint32_t wcnt[3];        // per-window append counters
    uint32_t hikey, lokey;   // key range of the candidate buffer
    float xmin;
    uint32_t nunique;        // unique history columns in this call's range
    uint32_t snap;
    uint32_t ncol;           // collected entries (multi-pass paths)
    uint32_t go;             // rows after which the consumers let the producer claim the next one
    uint32_t preq;           // passes over the current row requested from the producer
    uint32_t rst, rph;       // consumers' ring position between passes
    SelSlot sel[2];          // select results, alternating between passes
    // a second window collected with the top-p cut's window (the draw's, from
    // its predicted target): keys [b_klo, b_khi] in [slot0, b_n1) of the buffer
    uint32_t b_ok, b_klo, b_khi, b_n1;
    unsigned long long b_above, b_mass;
};

struct Smem {
    uint64_t* full;
    uint64_t* empty;
    uint64_t* rowfull;
    uint64_t* rowempty;
    RowCtl* ctl;
    uint64_t* red64;
    float* redf;
    uint32_t* red32;
    double* redd;
    uint32_t* blo;             // [2][NB] low words of the bin masses
    uint32_t* bhi;             // [2][NB] high words
    uint32_t* cnts;            // [2][NB]
    uint32_t* ckey;            // [CAND_CAP]
    uint32_t* cid;             // [CAND_CAP]
    uint32_t* bitmap;
    uint16_t* prefix;          // popcount of the bitmap before each 64-column pair of words
    uint32_t* counts;
    float* sval;
    uint32_t* scol;
    uint8_t* ring;
};

__host__ __device__ inline int align_up_i(int x, int a) { return (x + a - 1) / a * a; }

// Barriers + control block + reduction scratch; returns the first free offset.
__host__ __device__ inline int head_bytes(int nstage) {
    int o = 8 * (2 * nstage + 2 * RQ);
    o = align_up_i(o, 16) + (int)sizeof(RowCtl);
    o = align_up_i(o, 16) + (8 + 4 + 4 + 8) * NCW;
    return align_up_i(o, 128);
}

// The kernel's dynamic shared memory (every unsized extern __shared__ array
// starts at the same address).
extern __shared__ __align__(128) uint8_t fg_smem[];
// Its base, passed through an empty asm so the optimizer cannot hoist the
// pointers derived from it out of a loop: rebuilding the layout where it is
// used (a few integer adds from the grid-constant offsets) is cheaper than
// holding twenty 64-bit pointers live across the streaming loop.
__device__ __forceinline__ uint8_t* smem_base() {
    uint8_t* b = fg_smem;
    asm volatile("" : "+l"(b));
    return b;
}

// 32-bit shared-window address of the dynamic shared memory, opaque in the
// same way (one instruction where it is used).
__device__ __forceinline__ uint32_t smem_base32() {
    uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(fg_smem));
    asm volatile("" : "+r"(b));
    return b;
}
__host__ __device__ inline int ctl_offset(int nstage) { return align_up_i(8 * (2 * nstage + 2 * RQ), 16); }

__device__ __forceinline__ Smem carve(uint8_t* base, const KParams& P) {
    Smem s;
    s.full = reinterpret_cast<uint64_t*>(base);
    s.empty = s.full + P.nstage;
    s.rowfull = s.empty + P.nstage;
    s.rowempty = s.rowfull + RQ;
    int o = align_up_i(8 * (2 * P.nstage + 2 * RQ), 16);
    s.ctl = reinterpret_cast<RowCtl*>(base + o);
    o = align_up_i(o + (int)sizeof(RowCtl), 16);
    s.red64 = reinterpret_cast<uint64_t*>(base + o); o += 8 * NCW;
    s.redd = reinterpret_cast<double*>(base + o); o += 8 * NCW;
    s.redf = reinterpret_cast<float*>(base + o); o += 4 * NCW;
    s.red32 = reinterpret_cast<uint32_t*>(base + o);
    s.blo = reinterpret_cast<uint32_t*>(base + P.off_bins);
    s.bhi = s.blo + 2 * NB;
    s.cnts = reinterpret_cast<uint32_t*>(base + P.off_cnts);
    s.ckey = reinterpret_cast<uint32_t*>(base + P.off_ckey);
    s.cid = reinterpret_cast<uint32_t*>(base + P.off_cid);
    s.bitmap = reinterpret_cast<uint32_t*>(base + P.off_bitmap);
    s.prefix = reinterpret_cast<uint16_t*>(base + P.off_prefix);
    s.counts = reinterpret_cast<uint32_t*>(base + P.off_counts);
    s.sval = reinterpret_cast<float*>(base + P.off_sval);
    s.scol = reinterpret_cast<uint32_t*>(base + P.off_scol);
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
    const uintptr_t a0 = (reinterpret_cast<uintptr_t>(start) + 15) & ~uintptr_t(15);
    const uintptr_t a1 = reinterpret_cast<uintptr_t>(end) & ~uintptr_t(15);
    if (a1 <= a0) {
        g.interior = start; g.interior_bytes = 0; g.head = P.vocab; g.tail0 = P.vocab; g.ntiles = 0;
        return g;
    }
    g.interior = reinterpret_cast<const uint8_t*>(a0);
    g.interior_bytes = (int64_t)(a1 - a0);
    g.head = (int)((a0 - reinterpret_cast<uintptr_t>(start)) / ESZ);
    g.tail0 = g.head + (int)(g.interior_bytes / ESZ);
    g.ntiles = (int)((g.interior_bytes + TILE_BYTES - 1) / TILE_BYTES);
    return g;
}

// ---------------------------------------------------------------------------
// Per-row parameters (registers, identical in every consumer thread)
// ---------------------------------------------------------------------------
struct RowParams {
    int mode;
    int K;           // top-k (TOPK) or candidate target
    bool use_p;
    bool cand;       // candidate filter requested
    bool pen, freq_on, pres_on, rep_on;
    bool temp_on;    // y = x / T
    bool zsum;       // online sum-exp needed (NUCLEUS / FULL)
    float T, rT, top_p, rep, pres, freq, u;
    float c;         // log2(e) / T for the online sum-exp
    int bad;         // FG_ROW_BAD_PARAM / FG_ROW_BAD_UNIFORM
};

// Split path: the caller's row of launch row r, and the global id of the
// launch row's column 0.
__device__ __forceinline__ int src_row(const KParams& P, int r) { return P.nshard > 1 ? r / P.nshard : r; }
__device__ __forceinline__ int64_t col_base(const KParams& P, int r) {
    return P.vocab_offset + (P.nshard > 1 ? (int64_t)(r % P.nshard) * P.vocab : 0);
}

__device__ __forceinline__ RowParams row_params(const KParams& P, int r) {
    RowParams p;
    const int q = src_row(P, r);
    p.T = __ldg(P.temperature + q);
    p.top_p = __ldg(P.top_p + q);
    const int tk = __ldg(P.top_k + q);
    p.rep = P.rep ? __ldg(P.rep + q) : 1.0f;
    p.pres = P.pres ? __ldg(P.pres + q) : 0.0f;
    p.freq = P.freq ? __ldg(P.freq + q) : 0.0f;
    const bool g = P.greedy ? (__ldg(P.greedy + q) != 0) : false;
    p.u = __ldg(P.uniforms + q);
    p.bad = 0;
    // the merge samples values already divided by T
    if (P.merge_g > 0 && !g && p.T > 0.0f) p.T = 1.0f;
    const bool hist = P.pen_possible && (__ldg(P.hist_offsets + q + 1) > __ldg(P.hist_offsets + q));
    p.rep_on = hist && (p.rep != 1.0f);
    p.freq_on = hist && (p.freq != 0.0f);
    p.pres_on = hist && (p.pres != 0.0f);
    p.pen = p.rep_on || p.freq_on || p.pres_on;
    if (!(p.rep == p.rep) || !(p.pres == p.pres) || !(p.freq == p.freq)) p.bad |= FG_ROW_BAD_PARAM;
    p.zsum = false;
    if (g || p.T == 0.0f) {
        p.mode = MODE_GREEDY; p.K = 1; p.use_p = false; p.cand = false; p.temp_on = false;
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
    } else {
        p.mode = p.use_p ? MODE_NUCLEUS : MODE_FULL;
        // a shard of the split path keeps at most cand_max candidates
        p.K = (P.nshard > 1 && P.cand_max < K_NUCLEUS) ? P.cand_max : K_NUCLEUS;
        p.cand = true; p.zsum = true;
    }
    return p;
}

// Row queue: entries [0, B) hand out the rows that may need passes over the
// row after the stream (sampling rows whose top-k is off or above the
// candidate limit), entries [B, 2B) the other rows, so the long rows start
// first. Each entry belongs to the half that owns its row; a producer claims
// ROW_CLAIM entries per atomic. One: a claim of several entries could give one
// CTA two long rows to run back to back while other CTAs have none.
constexpr int ROW_CLAIM = 1;
__device__ __forceinline__ bool row_heavy(const KParams& P, int r) {
    const int q = src_row(P, r);
    const float T = __ldg(P.temperature + q);
    const bool g = P.greedy ? (__ldg(P.greedy + q) != 0) : false;
    const int tk = __ldg(P.top_k + q);
    if (g || T == 0.0f) return false;
    return tk <= 0 || tk > K_FAST_MAX;
}
// Fixup stage of the split path: only the rows the merge could not decide.
__device__ __forceinline__ bool row_wanted(const KParams& P, int r) {
    return P.redo == nullptr || (__ldg(P.redo + r) & FG_ROW_SPLIT_REDO) != 0;
}
__device__ __forceinline__ bool row_owned(const KParams& P, unsigned v) {
    const unsigned B = (unsigned)P.batch;
    if (v >= 2u * B) return false;
    return (v < B) == row_heavy(P, (int)(v % B));
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
    for (int steps = 0; steps < 8; ++steps) {
        if (k <= KEY_NEG_INF) return funkey(k);
        if (ydiv(p, funkey(k - 1)) >= yt) --k; else return funkey(k);
    }
    uint32_t lo = KEY_NEG_INF, hi = k;   // pred(hi) holds; smallest key where it holds
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo) / 2;
        if (ydiv(p, funkey(mid)) >= yt) hi = mid; else lo = mid + 1;
    }
    return funkey(hi);
}

// Smallest x with fkey(y(x)) >= yk (y is monotone in x). Starts from
// yk's value times T and walks a few keys; bisects over the key space if the
// walk is long. Identical in every thread (no barrier).
constexpr uint32_t KEY_POS_INF = 0xff800000u;
__device__ float x_lower(const RowParams& p, uint32_t yk) {
    if (yk <= KEY_NEG_INF) return -INFINITY;
    if (!p.temp_on) return funkey(yk);
    auto pred = [&](uint32_t k) { return fkey(ydiv(p, funkey(k))) >= yk; };
    if (yk > KEY_POS_INF || !pred(KEY_POS_INF)) return NAN;   // no such x
    const float g = funkey(yk) * p.T;
    uint32_t k = (g == g) ? fkey(g) : KEY_POS_INF;
    if (k < KEY_NEG_INF) k = KEY_NEG_INF;
    if (k > KEY_POS_INF) k = KEY_POS_INF;
    for (int steps = 0; steps < 8; ++steps) {
        if (pred(k)) {
            if (k <= KEY_NEG_INF || !pred(k - 1)) return funkey(k);
            --k;
        } else {
            ++k;   // k < KEY_POS_INF, where pred holds
        }
    }
    uint32_t lo = KEY_NEG_INF, hi = KEY_POS_INF;
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo) / 2;
        if (pred(mid)) hi = mid; else lo = mid + 1;
    }
    return funkey(lo);
}
// Largest x with fkey(y(x)) <= yk.
__device__ float x_upper(const RowParams& p, uint32_t yk) {
    if (yk >= KEY_POS_INF) return INFINITY;
    const float xn = x_lower(p, yk + 1u);
    if (!(xn == xn)) return INFINITY;
    const uint32_t kn = fkey(xn);
    return kn <= KEY_NEG_INF ? -INFINITY : funkey(kn - 1u);
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
__device__ __forceinline__ float cons_min_f(float v, const Smem& s, int tid) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((tid & 31) == 0) s.redf[tid >> 5] = v;
    csync();
    float r = s.redf[0];
#pragma unroll
    for (int w = 1; w < NCW; ++w) r = fminf(r, s.redf[w]);
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
// Exclusive prefix over consumer threads in thread order; returns excl, sets total.
__device__ __forceinline__ uint32_t cons_excl_scan_u32(uint32_t v, uint32_t& total, const Smem& s, int tid) {
    const int lane = tid & 31, w = tid >> 5;
    const uint32_t incl = warp_incl_scan_u32(v, lane);
    if (lane == 31) s.red32[w] = incl;
    csync();
    uint32_t base = 0, tot = 0;
#pragma unroll
    for (int i = 0; i < NCW; ++i) {
        const uint32_t t = s.red32[i];
        if (i < w) base += t;
        tot += t;
    }
    csync();
    total = tot;
    return base + incl - v;
}

// ---------------------------------------------------------------------------
// Histogram add: count, and (unless COUNT) a 64-bit weight as two 32-bit
// atomics with an exact carry (the returned old low word tells whether this
// addition wrapped). 64-bit shared-memory atomics are avoided: under contention
// they cost ~70x a 32-bit one on sm_100a.
// ---------------------------------------------------------------------------
template <bool COUNT>
__device__ __forceinline__ void add_bin(uint32_t* cnts, uint32_t* blo, uint32_t* bhi, bool valid, uint32_t d,
                                        uint64_t w) {
    if (!valid) return;
    reds_add(&cnts[d], 1u);
    if (COUNT || w == 0) return;
    const uint32_t l = (uint32_t)w;
    uint32_t h = (uint32_t)(w >> 32);
    if (l) {
        const uint32_t old = atoms_add(&blo[d], l);
        h += (old + l < old) ? 1u : 0u;
    }
    if (h) reds_add(&bhi[d], h);
}
__device__ __forceinline__ uint64_t bin_mass(const uint32_t* blo, const uint32_t* bhi, int d) {
    return ((uint64_t)bhi[d] << 32) | blo[d];
}

// ---------------------------------------------------------------------------
// Block radix select with 8-bit digits.
//
// Over the (key, weight) pairs every consumer thread yields through
// `enumerate` — enumerate(f) calls f(valid, key, weight) the same number of
// times in every lane of a warp — find key k* with
//     W(before k*) <= target < W(before k*) + W(at k*),
// "before" meaning larger keys (DESC) or smaller keys (ASC). Keys are known to
// share their top (32 - rem) bits with `prefix`. Weights are summed exactly in
// integers, so the result does not depend on thread scheduling. COUNT selects
// ignore the weight and count elements. ok=false when target >= total.
// ---------------------------------------------------------------------------
struct SelOut {
    uint32_t key;
    uint64_t before;   // weight strictly before key*
    uint64_t at;       // weight at key*
    uint32_t n_at;     // elements at key*
    bool ok;
};

// Number of low bits that vary among keys in [lo, hi].
__device__ __forceinline__ int varying_bits(uint32_t lo, uint32_t hi) {
    const uint32_t d = lo ^ hi;
    return d == 0 ? 0 : 32 - __clz(d);
}

// Block-wide inclusive scan over the NCT threads (thread order).
__device__ __forceinline__ uint64_t block_incl_scan_u64(uint64_t v, const Smem& s, int tid) {
    const int lane = tid & 31, wid = tid >> 5;
    uint64_t incl = warp_incl_scan_u64(v, lane);
    if (lane == 31) s.red64[wid] = incl;
    csync();
    uint64_t base = 0;
#pragma unroll
    for (int i = 0; i < NCW; ++i) if (i < wid) base += s.red64[i];
    return incl + base;
}

// Warp 0 scans the nb-bin histogram (nb <= NB) in (DESC ? descending :
// ascending) digit order and writes, to sel[slot], the digit whose bin holds
// `rel` (ok = 0 when rel >= total). Lane l owns scan positions [8l, 8l + 8).
template <bool DESC, bool COUNT>
__device__ __forceinline__ void warp0_scan_bins(const Smem& s, const uint32_t* cn, const uint32_t* bl,
                                                const uint32_t* bh, int nb, uint64_t rel, int slot, int lane) {
    uint64_t v[8];
    uint64_t lsum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int o = lane * 8 + j;
        const int d = DESC ? nb - 1 - o : o;
        v[j] = (o < nb) ? (COUNT ? (uint64_t)cn[d] : bin_mass(bl, bh, d)) : 0ull;
        lsum += v[j];
    }
    const uint64_t incl = warp_incl_scan_u64(lsum, lane);
    const uint64_t excl = incl - lsum;
    const bool mine = (excl <= rel) && (rel < incl);
    const uint32_t bal = __ballot_sync(0xffffffffu, mine);
    SelSlot& o = s.ctl->sel[slot];
    if (bal == 0) {
        if (lane == 0) o.ok = 0;
    } else if (lane == __ffs(bal) - 1) {
        uint64_t c = excl;
        int jj = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (jj == j && rel >= c + v[j]) { c += v[j]; jj = j + 1; }
        }
        if (jj > 7) jj = 7;
        const int d = DESC ? nb - 1 - (lane * 8 + jj) : lane * 8 + jj;
        o.ok = 1; o.digit = (uint32_t)d; o.before = c; o.nat = cn[d];
        o.at = COUNT ? (uint64_t)cn[d] : bin_mass(bl, bh, d);
    }
}

template <bool DESC, bool COUNT, class Enum>
__device__ SelOut block_select(Enum&& enumerate, uint64_t target, uint32_t prefix, int rem, const Smem& s,
                               int tid) {
    const int lane = tid & 31;
    (void)lane;
    SelOut out;
    uint32_t pmask = rem >= 32 ? 0u : ~((1u << rem) - 1u);
    prefix &= pmask;
    if (rem == 0) {
        uint64_t wsum = 0, csum = 0;
        enumerate([&](bool valid, uint32_t k, uint64_t wt) {
            if (valid && k == prefix) { ++csum; if (!COUNT) wsum += wt; }
        });
        const uint64_t nat = cons_sum_u64(csum, s, tid);
        const uint64_t W = COUNT ? nat : cons_sum_u64(wsum, s, tid);
        out.key = prefix; out.before = 0; out.at = W; out.n_at = (uint32_t)nat; out.ok = target < W;
        return out;
    }
    uint64_t before = 0, at = 0;
    uint32_t nat = 0;
    bool ok = true;
    int buf = 0, pass = 0;
    s.cnts[tid] = 0u;
    if (!COUNT) { s.blo[tid] = 0u; s.bhi[tid] = 0u; }
    csync();
    while (rem > 0) {
        const int w = rem < 8 ? rem : 8;
        const int shift = rem - w;
        const uint32_t dmask = (1u << w) - 1u;
        uint32_t* cn = s.cnts + buf * NB;
        uint32_t* bl = s.blo + buf * NB;
        uint32_t* bh = s.bhi + buf * NB;
        // clear the other buffer for the next pass (it was last read before the
        // previous pass's second barrier)
        s.cnts[(buf ^ 1) * NB + tid] = 0u;
        if (!COUNT) { s.blo[(buf ^ 1) * NB + tid] = 0u; s.bhi[(buf ^ 1) * NB + tid] = 0u; }
        enumerate([&](bool valid, uint32_t k, uint64_t wt) {
            const bool v = valid && ((k & pmask) == prefix);
            add_bin<COUNT>(cn, bl, bh, v, (k >> shift) & dmask, wt);
        });
        csync();
        if (tid < 32) warp0_scan_bins<DESC, COUNT>(s, cn, bl, bh, 1 << w, target - before, pass & 1, lane);
        csync();
        const SelSlot r = s.ctl->sel[pass & 1];
        if (!r.ok) { ok = false; break; }
        before += r.before;
        nat = r.nat; at = r.at;
        prefix |= r.digit << shift;
        pmask |= dmask << shift;
        rem = shift;
        buf ^= 1; ++pass;
    }
    out.key = prefix; out.before = before; out.at = at; out.n_at = nat; out.ok = ok;
    csync();   // every thread has read the last result slot before the next select writes it
    return out;
}

}  // namespace fg
