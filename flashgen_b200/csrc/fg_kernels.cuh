// fg_kernels.cuh — kernels behind the C ABI in include/flashgen_sampler.h.
//
//   fg_sample_kernel<DT>      one persistent CTA per row: fused penalties /
//                             temperature / top-k, launched by
//                             fg_sample_candidates (the local stage of
//                             vocabulary-sharded sampling). fg_sample itself
//                             runs the batch kernels (fg_stream.cuh) and the
//                             cluster kernel (fg_cluster.cuh). The kernel's
//                             shard / merge / fixup stages (KParams nshard,
//                             merge_g, redo) served an earlier small-batch
//                             path and are not launched by any entry point.
//   fg_argmax_kernel<DT>      row argmax (torch.argmax semantics)
//   fg_rep_penalty_kernel<DT> in-place repetition penalty
#pragma once
#include "fg_sample_kernel.cuh"

namespace fg {

constexpr float L2E = 1.4426950408889634f;

__device__ __forceinline__ float ex2_approx(float v) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(v));
    return y;
}

// ---------------------------------------------------------------------------
// Chunk helpers (one 16-byte chunk = VEC elements)
// ---------------------------------------------------------------------------
template <int DT> struct Neg;  // 16-byte pattern of -inf elements
template <> struct Neg<FG_DTYPE_F32> { static constexpr uint32_t W = 0xFF800000u; };
template <> struct Neg<FG_DTYPE_F16> { static constexpr uint32_t W = 0xFC00FC00u; };
template <> struct Neg<FG_DTYPE_BF16> { static constexpr uint32_t W = 0xFF80FF80u; };

__device__ __forceinline__ uint32_t word_get(const uint4& v, int q) {
    return q == 0 ? v.x : (q == 1 ? v.y : (q == 2 ? v.z : v.w));
}
template <int DT>
__device__ __forceinline__ float elem_get(const uint4& v, int e) {
    if constexpr (DT == FG_DTYPE_F32) {
        return __uint_as_float(word_get(v, e));
    } else {
        const uint32_t w = word_get(v, e >> 1);
        const uint16_t h = (e & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xffffu);
        if constexpr (DT == FG_DTYPE_BF16) return __uint_as_float(uint32_t(h) << 16);
        else return __half2float(__ushort_as_half(h));
    }
}
// Element e of a chunk set to -inf. Written as selects on the four words: a
// reference to a word chosen at run time would force the chunk (and with it
// the tile's registers) into local memory.
template <int DT>
__device__ __forceinline__ void elem_mask(uint4& v, int e) {
    if constexpr (DT == FG_DTYPE_F32) {
        constexpr uint32_t W = Neg<DT>::W;
        v.x = e == 0 ? W : v.x;
        v.y = e == 1 ? W : v.y;
        v.z = e == 2 ? W : v.z;
        v.w = e == 3 ? W : v.w;
    } else {
        const int q = e >> 1;
        const uint32_t keep = (e & 1) ? 0x0000ffffu : 0xffff0000u;
        const uint32_t neg = Neg<DT>::W & ~keep;
        v.x = q == 0 ? ((v.x & keep) | neg) : v.x;
        v.y = q == 1 ? ((v.y & keep) | neg) : v.y;
        v.z = q == 2 ? ((v.z & keep) | neg) : v.z;
        v.w = q == 3 ? ((v.w & keep) | neg) : v.w;
    }
}

// NaN-propagating max over CPT chunks (pairwise tree; packed pairs for 16-bit types).
template <int DT>
__device__ __forceinline__ float chunk_max1(const uint4& v) {
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
template <int DT>
__device__ __forceinline__ float chunks_max(const uint4 (&v)[CPT]) {
    float m = chunk_max1<DT>(v[0]);
#pragma unroll
    for (int j = 1; j < CPT; ++j) m = fmax_nan(m, chunk_max1<DT>(v[j]));
    return m;
}
// Minimum over CPT chunks (NaN ignored by fminf).
template <int DT>
__device__ __forceinline__ float chunks_min(const uint4 (&v)[CPT]) {
    float r = INFINITY;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
        if constexpr (DT == FG_DTYPE_F32) {
            r = fminf(r, fminf(fminf(__uint_as_float(v[j].x), __uint_as_float(v[j].y)),
                               fminf(__uint_as_float(v[j].z), __uint_as_float(v[j].w))));
        } else if constexpr (DT == FG_DTYPE_BF16) {
            const __nv_bfloat162 m = __hmin2(__hmin2(*reinterpret_cast<const __nv_bfloat162*>(&v[j].x),
                                                     *reinterpret_cast<const __nv_bfloat162*>(&v[j].y)),
                                             __hmin2(*reinterpret_cast<const __nv_bfloat162*>(&v[j].z),
                                                     *reinterpret_cast<const __nv_bfloat162*>(&v[j].w)));
            r = fminf(r, fminf(__low2float(m), __high2float(m)));
        } else {
            const __half2 m = __hmin2(__hmin2(*reinterpret_cast<const __half2*>(&v[j].x), *reinterpret_cast<const __half2*>(&v[j].y)),
                                      __hmin2(*reinterpret_cast<const __half2*>(&v[j].z), *reinterpret_cast<const __half2*>(&v[j].w)));
            r = fminf(r, fminf(__low2float(m), __high2float(m)));
        }
    }
    return r;
}

// Bit e set when element e of the chunk is >= xmin. For the 16-bit types
// x2 holds xmin rounded up to the type, in both halves: for a 16-bit x,
// x >= xmin exactly when x >= that value, so one packed compare tests two
// elements. NaN compares false.
template <int DT>
__device__ __forceinline__ uint32_t chunk_ge(const uint4& v, float xmin, uint32_t x2) {
    if constexpr (DT == FG_DTYPE_F32) {
        return (uint32_t)(__uint_as_float(v.x) >= xmin) | ((uint32_t)(__uint_as_float(v.y) >= xmin) << 1) |
               ((uint32_t)(__uint_as_float(v.z) >= xmin) << 2) | ((uint32_t)(__uint_as_float(v.w) >= xmin) << 3);
    } else {
        uint32_t m[4];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if constexpr (DT == FG_DTYPE_BF16)
                m[q] = __hge2_mask(*reinterpret_cast<const __nv_bfloat162*>(&w[q]),
                                   *reinterpret_cast<const __nv_bfloat162*>(&x2));
            else
                m[q] = __hge2_mask(*reinterpret_cast<const __half2*>(&w[q]), *reinterpret_cast<const __half2*>(&x2));
        }
        uint32_t b = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) b |= ((m[q] & 1u) | ((m[q] >> 15) & 2u)) << (2 * q);
        return b;
    }
}
template <int DT>
__device__ __forceinline__ uint32_t xmin_pair(float xmin) {
    if constexpr (DT == FG_DTYPE_BF16) {
        const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_ru(xmin));
        return h | (h << 16);
    } else if constexpr (DT == FG_DTYPE_F16) {
        const uint32_t h = __half_as_ushort(__float2half_ru(xmin));
        return h | (h << 16);
    } else {
        return 0u;
    }
}

// z += sum_e 2^(x_e * c - zmc) over every element of the chunks (two accumulators).
template <int DT>
__device__ __forceinline__ void chunks_sumexp(const uint4 (&v)[CPT], float c, float nzmc, float& z0, float& z1) {
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t w = word_get(v[j], q);
            if constexpr (DT == FG_DTYPE_F32) {
                if (q & 1) z1 += ex2_approx(__fmaf_rn(__uint_as_float(w), c, nzmc));
                else z0 += ex2_approx(__fmaf_rn(__uint_as_float(w), c, nzmc));
            } else {
                float lo, hi;
                if constexpr (DT == FG_DTYPE_BF16) {
                    lo = __uint_as_float(w << 16); hi = __uint_as_float(w & 0xffff0000u);
                } else {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
                    lo = f.x; hi = f.y;
                }
                z0 += ex2_approx(__fmaf_rn(lo, c, nzmc));
                z1 += ex2_approx(__fmaf_rn(hi, c, nzmc));
            }
        }
    }
}

// ---------------------------------------------------------------------------
// History prologue: bitmap of this row's history columns, the ascending list
// of distinct history columns (scol), a popcount prefix per 64-column pair of
// bitmap words (so a column's rank — its index in scol — costs three shared
// loads), and per-rank counts when a frequency penalty is set.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t hist_rank(const Smem& s, uint32_t c) {
    const uint32_t w = c >> 5;
    uint32_t r = s.prefix[w >> 1] + __popc(s.bitmap[w] & ((1u << (c & 31)) - 1u));
    if (w & 1u) r += __popc(s.bitmap[w - 1]);
    return r;
}

__device__ void history_prologue(const KParams& P, const Smem& s, const RowParams& p, int r, int tid) {
    const int nw = P.nwords;
    const int npair = (nw + 1) >> 1;
    const int lane = tid & 31;
    for (int w = tid; w < nw; w += NCT) s.bitmap[w] = 0u;
    csync();
    const int q = src_row(P, r);
    const int64_t h0 = __ldg(P.hist_offsets + q), h1 = __ldg(P.hist_offsets + q + 1);
    const int64_t cb = col_base(P, r);
    constexpr int HB = 4;        // ids per thread per batch, loaded together
    constexpr int HOWN = 4 * HB; // first-setters remembered in registers (histories <= NCT * HOWN)
    int bad = 0;
    // the thread whose atomicOr sets a column's bit first owns the column: it
    // writes the column's entry of the ascending list once the ranks are known
    uint32_t own_col[HOWN];
    uint32_t owned = 0u;
    int bi = 0;
    // the next batch's ids are loaded before this batch's bitmap atomics, so
    // one global-load latency is paid per history rather than per batch
    int32_t nxt[HB];
#pragma unroll
    for (int j = 0; j < HB; ++j) {
        const int64_t i = h0 + tid + (int64_t)j * NCT;
        nxt[j] = i < h1 ? __ldg(P.hist_ids + i) : -1;
    }
    for (int64_t b0 = h0; b0 < h1; b0 += (int64_t)NCT * HB, ++bi) {
        int32_t ids[HB];
#pragma unroll
        for (int j = 0; j < HB; ++j) {
            ids[j] = nxt[j];
            const int64_t i = b0 + (int64_t)NCT * HB + tid + (int64_t)j * NCT;
            nxt[j] = i < h1 ? __ldg(P.hist_ids + i) : -1;
        }
#pragma unroll
        for (int j = 0; j < HB; ++j) {
            const int64_t i = b0 + tid + (int64_t)j * NCT;
            if (i >= h1) continue;
            const int64_t gid = ids[j];
            if (gid < 0 || gid >= P.vocab_total) { bad = 1; continue; }
            const int64_t c = gid - cb;
            if (c >= 0 && c < P.vocab) {
                const uint32_t bit = 1u << (c & 31);
                if (!(s.bitmap[c >> 5] & bit)) {
                    const uint32_t old = atoms_or(&s.bitmap[c >> 5], bit);
                    if (!(old & bit) && bi * HB + j < HOWN) {
#pragma unroll
                        for (int q = 0; q < HOWN; ++q)
                            if (q == bi * HB + j) own_col[q] = (uint32_t)c;
                        owned |= 1u << (bi * HB + j);
                    }
                }
            }
        }
    }
    const bool own_all = (h1 - h0) <= (int64_t)NCT * HOWN;
    if (bad) reds_or(reinterpret_cast<uint32_t*>(&s.ctl->status), (uint32_t)FG_ROW_BAD_HISTORY);
    csync();
    // popcount prefix per 64-column pair of words, in pair order: warp w owns
    // pairs [w * ppw, (w + 1) * ppw), its lanes take 32 consecutive pairs at a
    // time (two-way bank conflicts at most)
    const int ppw = (npair + NCW - 1) / NCW;
    const int wq0 = (tid >> 5) * ppw, wq1 = min(npair, wq0 + ppw);
    auto pair_pop = [&](int q) -> uint32_t {
        if (q >= wq1) return 0u;
        return __popc(s.bitmap[2 * q]) + (2 * q + 1 < nw ? __popc(s.bitmap[2 * q + 1]) : 0);
    };
    uint32_t wsum = 0;
    for (int q0 = wq0; q0 < wq1; q0 += 32) wsum += pair_pop(q0 + lane);
    wsum = __reduce_add_sync(0xffffffffu, wsum);
    if (lane == 0) s.red32[tid >> 5] = wsum;
    csync();
    uint32_t run = 0, total = 0;
#pragma unroll
    for (int i = 0; i < NCW; ++i) {
        const uint32_t c = s.red32[i];
        if (i < (tid >> 5)) run += c;
        total += c;
    }
    csync();
    const uint32_t cap = (uint32_t)P.hu_cap;
    for (int q0 = wq0; q0 < wq1; q0 += 32) {
        const int q = q0 + lane;
        const uint32_t c = pair_pop(q);
        const uint32_t incl = warp_incl_scan_u32(c, lane);
        if (q < wq1) s.prefix[q] = (uint16_t)(run + incl - c);
        run += __shfl_sync(0xffffffffu, incl, 31);
    }
    csync();
    // ascending list of distinct columns: each owner writes its columns' entries
    // (histories longer than NCT * HOWN: words strided over the threads)
    if (own_all) {
#pragma unroll
        for (int q = 0; q < HOWN; ++q) {
            if ((owned >> q) & 1u) {
                const uint32_t rk = hist_rank(s, own_col[q]);
                if (rk < cap) s.scol[rk] = own_col[q];
            }
        }
    } else {
        for (int w = tid; w < nw; w += NCT) {
            uint32_t bits = s.bitmap[w];
            if (bits == 0u) continue;
            uint32_t rk = hist_rank(s, (uint32_t)(w * 32));
            while (bits) {
                const int b = __ffs(bits) - 1;
                bits &= bits - 1;
                if (rk < cap) s.scol[rk] = (uint32_t)(w * 32 + b);
                ++rk;
            }
        }
    }
    const uint32_t U = min(total, cap);
    if (tid == 0) {
        s.ctl->nunique = U;
        if (total > cap || total > 65535u) reds_or(reinterpret_cast<uint32_t*>(&s.ctl->status), (uint32_t)FG_ROW_BAD_PARAM);
    }
    for (uint32_t i = tid; i < U; i += NCT) s.sval[i] = -INFINITY;
    if (p.freq_on) {
        for (uint32_t i = tid; i < U; i += NCT) s.counts[i] = 0u;
        csync();
        for (int64_t b0 = h0; b0 < h1; b0 += (int64_t)NCT * HB) {
            int32_t ids[HB];
#pragma unroll
            for (int j = 0; j < HB; ++j) {
                const int64_t i = b0 + tid + (int64_t)j * NCT;
                ids[j] = i < h1 ? __ldg(P.hist_ids + i) : -1;
            }
#pragma unroll
            for (int j = 0; j < HB; ++j) {
                const int64_t i = b0 + tid + (int64_t)j * NCT;
                const int64_t gid = ids[j];
                const int64_t c = gid - cb;
                bool v = i < h1 && gid >= 0 && gid < P.vocab_total && c >= 0 && c < P.vocab;
                const uint32_t rk = v ? hist_rank(s, (uint32_t)c) : 0u;
                v = v && rk < U;
                if (v) reds_add(&s.counts[rk], 1u);
            }
        }
    }
    csync();
}

// Penalised value of the history column with the given rank.
__device__ __forceinline__ float penalize(const RowParams& p, const Smem& s, uint32_t rank, float x) {
    if (p.rep_on) x = (x > 0.0f) ? __fdiv_rn(x, p.rep) : __fmul_rn(x, p.rep);
    if (p.freq_on) x = __fsub_rn(x, __fmul_rn(p.freq, (float)s.counts[rank]));
    if (p.pres_on) x = __fsub_rn(x, p.pres);
    return x;
}
// History bits of columns [c0, c0 + n), n <= 8.
__device__ __forceinline__ uint32_t hist_bits(const Smem& s, int nwords, int c0, int n) {
    const int w = c0 >> 5, b = c0 & 31;
    const uint32_t lo = s.bitmap[w];
    const uint32_t hi = (b + n > 32 && w + 1 < nwords) ? s.bitmap[w + 1] : 0u;
    return __funnelshift_r(lo, hi, b) & ((1u << n) - 1u);
}

// ---------------------------------------------------------------------------
// Per-thread streaming state
// ---------------------------------------------------------------------------
struct Stream {
    float tmax;           // NaN-propagating max of penalised x (whole row)
    float imax;           // max over the streamed interior (greedy rows)
    int itile;            // first tile where imax was reached
    float tmin;           // min over the row (rows with a sum-exp)
    float zm, nzmc;       // running max for the sum-exp and -fl(zm * c)
    float z0, z1;         // sum of 2^(x*c + nzmc)
    float xmin;           // register copy of the candidate filter
    float bestv;          // greedy rows: best element outside the streamed interior
    uint32_t bestc;
    bool cand;
    uint32_t base;        // candidates before the current window
    uint32_t win;         // window index (counter slot = win % 3)
    uint32_t khi, klo;    // key range of this thread's appends
};

// Append one candidate (no warp collectives: 32-bit shared atomics on one
// counter are combined by the hardware). The key range is tracked per thread
// and reduced only when a compaction needs it.
__device__ __forceinline__ void append1(const Smem& s, Stream& st, uint32_t key, uint32_t col) {
    const int slot = (int)(st.win % 3u);
    const uint32_t pos = st.base + atoms_add(&s.ctl->wcnt[slot], 1u);
    if (pos < (uint32_t)CAND_CAP) { s.ckey[pos] = key; s.cid[pos] = col; } else s.ctl->ovf[slot] = 1;
    st.khi = max(st.khi, key); st.klo = min(st.klo, key);
}

// One element outside the streamed interior (ragged columns, merged history).
__device__ __forceinline__ void process_one(const RowParams& p, const Smem& s, Stream& st, float x,
                                            uint32_t col, bool valid, int lane) {
    if (valid) {
        st.tmax = fmax_nan(st.tmax, x);
        if (p.mode == MODE_GREEDY && (x > st.bestv || (x == st.bestv && col < st.bestc))) { st.bestv = x; st.bestc = col; }
        if (p.zsum) {
            st.tmin = fminf(st.tmin, x);
            if (x > st.zm) {
                const float nn = -(x * p.c);
                const float f = ex2_approx(nn - st.nzmc);
                st.z0 *= f; st.z1 *= f;
                st.zm = x; st.nzmc = nn;
            }
            st.z0 += ex2_approx(__fmaf_rn(x, p.c, st.nzmc));
        }
    }
    if (st.cand && valid && x >= st.xmin) append1(s, st, fkey(x), col);
}

// ---------------------------------------------------------------------------
// Compaction: exact K-th largest candidate key -> xmin; drop keys below it
// (stable, in place). Returns the new candidate count.
// ---------------------------------------------------------------------------
// Order-preserving 16-bit keys of unpenalised 16-bit logits (key16 order ==
// key order), and back. bf16: the top half of the 32-bit key (its low half is
// 0x0000 for positive values, 0xffff for negative ones). fp16: the key of the
// half's own bit pattern.
__device__ __forceinline__ uint32_t key16_of(uint32_t k, int dt16) {
    if (dt16 == FG_DTYPE_BF16) return k >> 16;
    const uint32_t h = __half_as_ushort(__float2half_rn(funkey(k)));
    return (h & 0x8000u) ? (~h & 0xffffu) : (h | 0x8000u);
}
__device__ __forceinline__ uint32_t key_from16(uint32_t k16, int dt16) {
    if (dt16 == FG_DTYPE_BF16) return (k16 << 16) | ((k16 & 0x8000u) ? 0u : 0xffffu);
    const uint32_t h = (k16 & 0x8000u) ? (k16 & 0x7fffu) : (~k16 & 0xffffu);
    return fkey(__half2float(__ushort_as_half((unsigned short)h)));
}

// Block min and max of a u32 in one barrier round.
__device__ __forceinline__ void cons_minmax_u32(uint32_t& mn, uint32_t& mx, const Smem& s, int tid) {
    mn = __reduce_min_sync(0xffffffffu, mn);
    mx = __reduce_max_sync(0xffffffffu, mx);
    if ((tid & 31) == 0) { s.red32[tid >> 5] = mn; reinterpret_cast<uint32_t*>(s.redf)[tid >> 5] = mx; }
    csync();
    uint32_t a = s.red32[0], b = reinterpret_cast<const uint32_t*>(s.redf)[0];
#pragma unroll
    for (int w = 1; w < NCW; ++w) { a = min(a, s.red32[w]); b = max(b, reinterpret_cast<const uint32_t*>(s.redf)[w]); }
    csync();
    mn = a; mx = b;
}

// ---------------------------------------------------------------------------
// Compaction: exact K-th largest candidate key -> xmin; drop keys below it.
// dt16 (FG_DTYPE_BF16 / FG_DTYPE_F16, else 0): every candidate is an
// unpenalised 16-bit logit, so the select runs on 16-bit keys (two 8-bit
// passes). The kept entries are
// rewritten in any order (nothing downstream depends on it): every thread
// holds its CAND_CAP / NCT entries in registers, then writes the kept ones at
// positions from one atomic per warp. Returns the new candidate count.
// ---------------------------------------------------------------------------
__device__ uint32_t compact(const RowParams& p, const Smem& s, int tid, uint32_t n, Stream& st, int dt16) {
    static_assert(CAND_CAP % NCT == 0, "entries per thread");
    constexpr int PER = CAND_CAP / NCT;
    RowCtl* ctl = s.ctl;
    if (n <= (uint32_t)p.K) return n;
    uint32_t lo = st.klo, hi = st.khi;
    cons_minmax_u32(lo, hi, s, tid);
    if (lo > hi) return n;
    if (tid == 0) ctl->ncol = 0u;
    auto kx = [&](uint32_t k) { return dt16 ? key16_of(k, dt16) : k; };
    const uint32_t lo_x = kx(lo), hi_x = kx(hi);
    const SelOut so = block_select<true, true>(
        [&](auto&& f) {
            for (uint32_t i0 = 0; i0 < n; i0 += NCT) {
                const uint32_t i = i0 + tid;
                f(i < n, i < n ? kx(s.ckey[i]) : 0u, 1ull);
            }
        },
        (uint64_t)(p.K - 1), lo_x, varying_bits(lo_x, hi_x), s, tid);
    if (!so.ok) return n;
    if (tid == 0) {
        const float xm = xmin_for(p, funkey(dt16 ? key_from16(so.key, dt16) : so.key));
        if (xm > ctl->xmin) ctl->xmin = xm;
    }
    uint32_t kk[PER], ii[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const uint32_t idx = (uint32_t)(j * NCT + tid);
        kk[j] = idx < n ? s.ckey[idx] : 0u;
        ii[j] = idx < n ? s.cid[idx] : 0u;
    }
    csync();   // every entry is in registers and xmin is published
    const uint32_t kmin = fkey(ctl->xmin);
    st.klo = max(st.klo, kmin);
    uint32_t cnt = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) cnt += ((uint32_t)(j * NCT + tid) < n && kk[j] >= kmin) ? 1u : 0u;
    const int lane = tid & 31;
    const uint32_t incl = warp_incl_scan_u32(cnt, lane);
    uint32_t base = 0;
    if (lane == 31) base = atoms_add(&ctl->ncol, incl);
    base = __shfl_sync(0xffffffffu, base, 31) + incl - cnt;
#pragma unroll
    for (int j = 0; j < PER; ++j)
        if ((uint32_t)(j * NCT + tid) < n && kk[j] >= kmin) { s.ckey[base] = kk[j]; s.cid[base] = ii[j]; ++base; }
    csync();
    return ctl->ncol;
}

// End of a candidate window, without any call (the streaming loop must not
// contain one): uniform candidate count, overflow, and whether the buffer must
// be compacted before the next window (it passed `limit`, or the next tile
// could overflow it at twice this window's append rate). Sets st.base to the
// count and rate2 to twice this window's appends.
__device__ __forceinline__ bool window_end(uint32_t a_ctl, int tid, Stream& st, uint32_t limit, uint32_t kcap,
                                           uint64_t& rate2) {
    csync();
    const uint32_t slot = st.win % 3u;
    const uint32_t n = st.base + lds_u32(a_ctl + (uint32_t)offsetof(RowCtl, wcnt) + 4u * slot);
    const bool ovf = lds_u32(a_ctl + (uint32_t)offsetof(RowCtl, ovf) + 4u * slot) != 0u;
    if (tid == 0) {
        const uint32_t nx = (slot + 2u) % 3u;
        sts_u32(a_ctl + (uint32_t)offsetof(RowCtl, wcnt) + 4u * nx, 0u);
        sts_u32(a_ctl + (uint32_t)offsetof(RowCtl, ovf) + 4u * nx, 0u);
    }
    st.win += 1;
    rate2 = 2ull * (uint64_t)(n - st.base);
    st.base = n;
    if (!st.cand) return false;
    if (ovf) { st.cand = false; return false; }
    return n > limit || n > kcap || (uint64_t)n + rate2 + 64ull > (uint64_t)CAND_CAP;
}
// Tiles (a power of two <= span_max) the next window may cover with n
// candidates at rate2 / span appends per tile.
__device__ __forceinline__ int window_span(uint32_t n, uint64_t rate2, int span, int span_max) {
    int next = span_max;
    const uint64_t sp = (uint64_t)(span > 0 ? span : 1);
    while (next > 1 && (uint64_t)n + rate2 * (uint64_t)next / sp + 64ull > (uint64_t)CAND_CAP) next >>= 1;
    return next;
}
__device__ __forceinline__ int span_max_at(int t) { return t < 4 ? 1 : (t < 16 ? 4 : 8); }

// End of a candidate window of `span` tiles: uniform candidate count, then a
// compaction when the buffer passed `limit` or when the next window could
// overflow it at twice this window's append rate. Returns the number of tiles
// (a power of two <= span_max) the next window may cover at that rate.
__device__ __forceinline__ uint32_t compact_cold(const KParams& P, int tid, int r, uint32_t n, uint32_t klo,
                                              uint32_t khi, int dt16) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    Stream st;
    st.klo = klo;
    st.khi = khi;
    return compact(p, s, tid, n, st, dt16);
}

__device__ __forceinline__ int window_check(const KParams& P, int r, const RowParams& p, const Smem& s, int tid,
                                           Stream& st, uint32_t limit, int span, int span_max) {
    csync();
    const int slot = (int)(st.win % 3u);
    uint32_t n = st.base + s.ctl->wcnt[slot];
    const bool ovf = s.ctl->ovf[slot] != 0;
    if (tid == 0) { s.ctl->wcnt[(slot + 2) % 3] = 0u; s.ctl->ovf[(slot + 2) % 3] = 0; }
    st.win += 1;
    int next = span_max;
    if (st.cand) {
        if (ovf) {
            st.cand = false;
        } else {
            const uint64_t rate2 = 2ull * (uint64_t)(n - st.base);   // twice the appends of this window
            auto fits = [&](uint32_t nn, int sp) {
                return (uint64_t)nn + rate2 * (uint64_t)sp / (uint64_t)(span > 0 ? span : 1) + 64ull <=
                       (uint64_t)CAND_CAP;
            };
            if (n > limit || !fits(n, 1)) {
                n = compact_cold(P, tid, r, n, st.klo, st.khi, 0);
                st.klo = max(st.klo, fkey(s.ctl->xmin));
                if (n > limit) st.cand = false;
            }
            while (next > 1 && !fits(n, next)) next >>= 1;
        }
        st.xmin = s.ctl->xmin;
    }
    st.base = n;
    return next;
}

// ---------------------------------------------------------------------------
// Whole-row enumeration from global memory (L2) for the multi-pass paths.
// f(col, x) with x the penalised fp32 value.
// ---------------------------------------------------------------------------
template <int DT, class F>
__device__ __forceinline__ void for_row(const KParams& P, const Smem& s, const RowParams& p, int r,
                                        const RowGeom& g, int tid, F&& f) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE, VEC = E::VEC;
    const uint8_t* row = reinterpret_cast<const uint8_t*>(P.logits) + (int64_t)r * P.row_stride * ESZ;
    const int nh = g.head, nt = P.vocab - g.tail0;
    if (tid < 32 && nh + nt > 0) {
        const bool valid = tid < nh + nt;
        const int c = tid < nh ? tid : g.tail0 + (tid - nh);
        float x = -INFINITY;
        if (valid) {
            x = E::load(row, c);
            if (p.pen && (hist_bits(s, P.nwords, c, 1) & 1u)) x = penalize(p, s, hist_rank(s, (uint32_t)c), x);
        }
        f(valid, valid ? c : 0, x);
    }
    // The interior comes through the ring: the producer streams the row once
    // more for each request (from L2, where rows that may need passes are kept
    // with an evict-last policy), with the copies of several tiles in flight.
    RowCtl* ctl = s.ctl;
    volatile int* abort = &ctl->abort;
    const uint32_t ns = (uint32_t)P.nstage;
    uint32_t st = ctl->rst, ph = ctl->rph;
    csync();   // every thread has the position before it moves
    if (tid == 0) { volatile uint32_t* q = &ctl->preq; *q = *q + 1u; }
    const int lane = tid & 31;
    for (int t = 0; t < g.ntiles; ++t) {
        const bool ok = mbar_wait(&s.full[st], ph, abort);
        if (!ok) *abort = 1;
        const int64_t left = g.interior_bytes - (int64_t)t * TILE_BYTES;
        const int nch = ok ? (int)((left < TILE_BYTES ? left : TILE_BYTES) / 16) : 0;
        const uint8_t* tile = s.ring + (int64_t)st * TILE_BYTES;
        uint4 v[CPT];
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            const int ch = tid + j * NCT;
            v[j] = ch < nch ? *reinterpret_cast<const uint4*>(tile + (int64_t)ch * 16) : make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[st]);
        if (++st == ns) { st = 0; ph ^= 1u; }
        const int tcol0 = g.head + t * (TILE_BYTES / ESZ);
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            const int ch = tid + j * NCT;
            const bool valid = ch < nch;
            float x[VEC];
            const int c0 = tcol0 + ch * VEC;
            if (valid) {
                E::unpack(v[j], x);
                if (p.pen) {
                    uint32_t bits = hist_bits(s, P.nwords, c0, VEC);
                    while (bits) {
                        const int e = __ffs(bits) - 1;
                        bits &= bits - 1;
                        const uint32_t rk = hist_rank(s, (uint32_t)(c0 + e));
#pragma unroll
                        for (int q = 0; q < VEC; ++q)
                            if (q == e) x[q] = penalize(p, s, rk, x[q]);
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < VEC; ++e) x[e] = -INFINITY;
            }
#pragma unroll
            for (int e = 0; e < VEC; ++e) f(valid, valid ? c0 + e : 0, x[e]);
        }
    }
    csync();   // every thread is past its reads of the position
    if (tid == 0) { ctl->rst = st; ctl->rph = ph; }
    csync();
}

__device__ __forceinline__ uint64_t q_of(float e, float scale) { return (uint64_t)__float2ull_rn(e * scale); }
// Fast mass of a value y outside the candidate set (a function of y alone, so
// equal values get equal masses).
__device__ __forceinline__ float efast(float y, float My) { return ex2_approx((y - My) * L2E); }

// ---------------------------------------------------------------------------
// Locate, over the region R of the row (elements whose y-key lies in
// [rlo, rhi]), the element where the cumulative fast mass in descending y
// order crosses `target` (clamped to the region's total).
//   level 0: NB bins linear in y over [ylo, yhi] (values at or below ylo,
//            whose masses are zero at this precision, share bin 0);
//   if the crossing bin holds more elements than the buffer can take, its key
//   range is refined with 8-bit radix passes;
//   the crossing set is collected into [slot0, CAND_CAP) and the element is
//   selected exactly among it.
// ---------------------------------------------------------------------------
struct Located {
    bool ok;
    bool in_buffer;    // the key's elements were collected into [n0, n1)
    uint32_t key;      // y-key of the element
    uint64_t before;   // region mass strictly above key
    uint64_t at;       // mass at key (all elements of that key)
    uint32_t n_at;
    uint64_t total;    // region mass
    uint32_t n0, n1;
};

template <int DT>
__device__ __forceinline__ Located locate(const KParams& P, const Smem& s, const RowParams& p, int r, const RowGeom& g, int tid,
                          uint32_t rlo, uint32_t rhi, float ylo, float yhi, uint64_t target, float My, float scale,
                          uint32_t slot0) {
    const int lane = tid & 31;
    Located L;
    L.ok = false; L.in_buffer = false; L.total = 0; L.n0 = slot0; L.n1 = slot0;
    if (rlo > rhi) return L;
    const float span = yhi - ylo;
    const float inv = (span > 0.0f && span < INFINITY) ? (float)NB / span : 0.0f;
    auto lbin = [&](float y) -> uint32_t {
        if (!(y > ylo)) return 0u;
        const float t = (y - ylo) * inv;
        return t >= (float)(NB - 1) ? (uint32_t)(NB - 1) : (uint32_t)t;
    };
    uint32_t* cn = s.cnts;
    uint32_t* bl = s.blo;
    uint32_t* bh = s.bhi;
    // ---- level 0: linear bins ----
    cn[tid] = 0u; bl[tid] = 0u; bh[tid] = 0u;
    csync();
    for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
        const float y = ydiv(p, x);
        const uint32_t k = fkey(y);
        const bool v = valid && k >= rlo && k <= rhi;
        add_bin<false>(cn, bl, bh, v, lbin(y), v ? q_of(efast(y, My), scale) : 0ull);
    });
    csync();
    L.total = cons_sum_u64(bin_mass(bl, bh, tid), s, tid);
    if (L.total == 0) return L;
    if (target >= L.total) target = L.total - 1;
    if (tid < 32) warp0_scan_bins<true, false>(s, cn, bl, bh, NB, target, 0, tid);
    csync();
    const SelSlot r0 = s.ctl->sel[0];
    csync();
    if (!r0.ok) return L;
    const uint32_t b0 = r0.digit;
    uint64_t before = r0.before;
    uint32_t cnt = r0.nat;
    const uint32_t room = slot0 < (uint32_t)CAND_CAP ? (uint32_t)CAND_CAP - slot0 : 0u;
    // ---- refine by key digits while the crossing set does not fit ----
    uint32_t prefix = 0u, pmask = 0u;
    int pass = 1;
    if (cnt > room) {
        uint32_t kmn = 0xffffffffu, kmx = 0u;
        for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
            const float y = ydiv(p, x);
            const uint32_t k = fkey(y);
            if (valid && k >= rlo && k <= rhi && lbin(y) == b0) { kmn = min(kmn, k); kmx = max(kmx, k); }
        });
        kmn = cons_min_u32(kmn, s, tid);
        kmx = cons_max_u32(kmx, s, tid);
        int rem = varying_bits(kmn, kmx);
        pmask = rem >= 32 ? 0u : ~((1u << rem) - 1u);
        prefix = kmn & pmask;
        if (rem == 0) {
            // every element of the crossing bin has one key; ids come from a row pass
            L.ok = true; L.key = kmn; L.before = before; L.at = r0.at; L.n_at = cnt;
            return L;
        }
        while (cnt > room && rem > 0) {
            const int w = rem < 8 ? rem : 8;
            const int shift = rem - w;
            const uint32_t dmask = (1u << w) - 1u;
            const int nb = 1 << w;
            cn[tid] = 0u; bl[tid] = 0u; bh[tid] = 0u;
            csync();
            for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
                const float y = ydiv(p, x);
                const uint32_t k = fkey(y);
                const bool v = valid && k >= rlo && k <= rhi && lbin(y) == b0 && (k & pmask) == prefix;
                add_bin<false>(cn, bl, bh, v, (k >> shift) & dmask, v ? q_of(efast(y, My), scale) : 0ull);
            });
            csync();
            if (tid < 32) warp0_scan_bins<true, false>(s, cn, bl, bh, nb, target - before, pass & 1, tid);
            csync();
            const SelSlot rr = s.ctl->sel[pass & 1];
            csync();
            ++pass;
            if (!rr.ok) return L;
            before += rr.before;
            prefix |= rr.digit << shift;
            pmask |= dmask << shift;
            rem = shift;
            cnt = rr.nat;
            if (cnt > room && rem == 0) {
                // every remaining element has this key; its ids are found with a row pass
                L.ok = true; L.key = prefix; L.before = before; L.at = rr.at; L.n_at = cnt;
                return L;
            }
        }
    }
    // ---- collect the crossing set ----
    if (tid == 0) s.ctl->ncol = 0u;
    csync();
    uint32_t kmn = 0xffffffffu, kmx = 0u;
    for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
        const float y = ydiv(p, x);
        const uint32_t k = fkey(y);
        if (valid && k >= rlo && k <= rhi && lbin(y) == b0 && (k & pmask) == prefix) {
            const uint32_t pos = slot0 + atoms_add(&s.ctl->ncol, 1u);
            if (pos < (uint32_t)CAND_CAP) { s.ckey[pos] = k; s.cid[pos] = (uint32_t)c; }
            kmn = min(kmn, k); kmx = max(kmx, k);
        }
    });
    kmn = cons_min_u32(kmn, s, tid);
    kmx = cons_max_u32(kmx, s, tid);
    const uint32_t n1 = min((uint32_t)CAND_CAP, slot0 + s.ctl->ncol);
    csync();
    const SelOut so = block_select<true, false>(
        [&](auto&& f) {
            for (uint32_t i0 = slot0; i0 < n1; i0 += NCT) {
                const uint32_t i = i0 + tid;
                const bool v = i < n1;
                const uint32_t k = v ? s.ckey[i] : 0u;
                f(v, k, v ? q_of(efast(funkey(k), My), scale) : 0ull);
            }
        },
        target - before, kmn, varying_bits(kmn, kmx), s, tid);
    L.ok = so.ok; L.in_buffer = true; L.key = so.key; L.before = before + so.before; L.at = so.at; L.n_at = so.n_at;
    L.n0 = slot0; L.n1 = n1;
    return L;
}

// ---------------------------------------------------------------------------
// Windowed locate: locate()'s contract at a fraction of its cost.
//
// It works on x (the penalised logit before temperature): y = x / T is
// monotone in x, so every region and window test is two float compares, and
// the exact division is only done for the few collected elements.
//   * A histogram pass only COUNTS elements per bin (one 32-bit shared atomic
//     each). NW bins are linear in x over the current window.
//   * A bin's mass lies between count * m(lower edge) and count * m(upper
//     edge); the edges are widened by the rounding slack of the bin function
//     and of y = x / T, and m by the error of the fast exponentials and of the
//     rounding to integers. The bins whose bracketed cumulative masses
//     straddle the target make the next window, which certainly holds the
//     crossing element. Window edges are closed under equal y, so a run of
//     tied values is never split.
//   * The mass above the window is summed exactly in registers, from
//     2^(x * log2e / T - My * log2e).
//   * When the window fits the free buffer its elements are collected with
//     their y-keys and the crossing element is selected exactly, with the
//     integer masses locate() gives elements of the candidate buffer.
// `fallback` is set when no window fits (a run of equal values longer than
// the free space) or a bracket is found violated.
// ---------------------------------------------------------------------------
constexpr int NW = 4 * NB;   // bins per level; the counts use the blo/bhi area (4 * NB words)
constexpr int WDEPTH = 3;    // histogram levels before the fallback

constexpr int NW0 = 2 * NW;  // level-0 bins when the free part of the candidate buffer can hold them

template <int NBIN>
__device__ __forceinline__ int wbin(float x, float xa, float inv) {
    const float t = (x - xa) * inv;
    if (!(t > 0.0f)) return 0;
    return t >= (float)(NBIN - 1) ? NBIN - 1 : (int)t;
}

struct WWin {
    int lo, hi;
    uint32_t count;
    bool any;
};

// One level: bins over [wl, wu] (x), counts in cnt. Returns the bins whose
// bracketed cumulative mass, descending from `above`, straddles T.
template <int NBIN>
__device__ WWin wscan(const Smem& s, const uint32_t* cnt, float wl, float wu, float inv, double sx,
                      const RowParams& p, float My, double scale, double above, double T, int tid) {
    constexpr int PER = NBIN / NCT;
    const int lane = tid & 31, wid = tid >> 5;
    const double w = inv > 0.0f ? 1.0 / (double)inv : 0.0;
    const double rT = p.temp_on ? 1.0 / (double)p.T : 1.0;
    double lq[PER], uq[PER];
    uint32_t c[PER];
    double sl = 0.0, su = 0.0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int b = NBIN - 1 - (tid * PER + j);   // thread order = descending bins
        c[j] = cnt[b];
        lq[j] = 0.0;
        uq[j] = 0.0;
        if (c[j]) {
            double e0 = (b == 0 || w == 0.0) ? (double)wl : (double)wl + (double)b * w - sx;
            double e1 = (b == NBIN - 1 || w == 0.0) ? (double)wu : (double)wl + (double)(b + 1) * w + sx;
            e0 = fmax(e0, (double)wl) * rT;
            e1 = fmin(e1, (double)wu) * rT;
            e0 -= fabs(e0) * 2.4e-7;   // y = fl(x / T)
            e1 += fabs(e1) * 2.4e-7;
            const double ml = floor(exp(e0 - (double)My) * scale * (1.0 - 3e-5)) - 1.0;
            const double mh = fmin(ceil(exp(e1 - (double)My) * scale * (1.0 + 3e-5)) + 1.0, 1e300);
            lq[j] = (double)c[j] * fmax(ml, 0.0);
            uq[j] = (double)c[j] * mh;
        }
        sl += lq[j];
        su += uq[j];
    }
    double il = sl, iu = su;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double tl = __shfl_up_sync(0xffffffffu, il, o);
        const double tu = __shfl_up_sync(0xffffffffu, iu, o);
        if (lane >= o) { il += tl; iu += tu; }
    }
    if (lane == 31) { s.redd[wid] = il; s.red64[wid] = (uint64_t)__double_as_longlong(iu); }
    csync();
    double bl = 0.0, bu = 0.0;
#pragma unroll
    for (int i = 0; i < NCW; ++i)
        if (i < wid) { bl += s.redd[i]; bu += __longlong_as_double((long long)s.red64[i]); }
    csync();
    double pl = bl + il - sl, pu = bu + iu - su;
    int bmax = -1, bmin = NBIN;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int b = NBIN - 1 - (tid * PER + j);
        const double exL = (above + pl) * (1.0 - 1e-12) - 2.0;
        const double inU = (above + pu + uq[j]) * (1.0 + 1e-12) + 2.0;
        if (c[j] && exL <= T && T < inU) { bmax = max(bmax, b); bmin = min(bmin, b); }
        pl += lq[j];
        pu += uq[j];
    }
    WWin out;
    const uint32_t hi1 = cons_max_u32((uint32_t)(bmax + 1), s, tid);
    const uint32_t lo = cons_min_u32((uint32_t)bmin, s, tid);
    out.any = hi1 > 0u;
    out.hi = (int)hi1 - 1;
    out.lo = (int)lo;
    uint64_t cc = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int b = NBIN - 1 - (tid * PER + j);
        if (out.any && b >= out.lo && b <= out.hi) cc += c[j];
    }
    out.count = (uint32_t)cons_sum_u64(cc, s, tid);
    return out;
}

// Exact mass of region R (y-keys in [rlo, rhi]), one row pass.
template <int DT>
__device__ __forceinline__ uint64_t region_mass(const KParams& P, const Smem& s, const RowParams& p, int r, const RowGeom& g,
                                int tid, uint32_t rlo, uint32_t rhi, float My, float scale) {
    uint64_t acc = 0;
    for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
        const float y = ydiv(p, x);
        const uint32_t k = fkey(y);
        if (valid && k >= rlo && k <= rhi) acc += q_of(efast(y, My), scale);
    });
    return cons_sum_u64(acc, s, tid);
}

struct WLoc {
    bool fallback;
    Located L;
};

// The passes of the windowed locate, each its own function with scalar
// arguments: the per-element loop then keeps its few values in registers
// instead of reloading the caller's spilled state for every element.
// Level-0 counts: NW0 bins in the candidate buffer's free part from slot0,
// else NW bins in the blo/bhi area.
template <int DT, int NBIN>
__device__ __noinline__ void wpass_count(const KParams& P, int tid, int r, float a0, float bi, float xlo, float xhi,
                                         uint32_t slot0) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    uint32_t* cnt = NBIN == NW0 ? s.ckey + slot0 : s.blo;
    for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
        if (valid && x >= a0 && x <= xhi && x >= xlo) reds_add(&cnt[wbin<NBIN>(x, a0, bi)], 1u);
    });
}
// Mass above the window (per thread), counts inside it. Branch-free per
// element: the mass is computed for every element and added under a
// predicate, so a warp does not run both paths.
template <int DT>
__device__ __noinline__ uint64_t wpass_mass(const KParams& P, int tid, int r, float a0, float a1, float bi, float xlo,
                                            float xhi, float cxx, float nmy, float scale) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    uint32_t* cnt = s.blo;
    uint64_t acc = 0;
    for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
        const bool inr = valid && x >= xlo && x <= xhi;
        const uint64_t q = q_of(ex2_approx(__fmaf_rn(x, cxx, nmy)), scale);
        acc += (inr && x > a1) ? q : 0ull;
        if (inr && x <= a1 && x >= a0) reds_add(&cnt[wbin<NW>(x, a0, bi)], 1u);
    });
    return acc;
}
struct WRun { uint64_t acc, cnt; };
// Mass above a run of equal values [a0, a1] and its length (per thread).
template <int DT>
__device__ __noinline__ WRun wpass_run(const KParams& P, int tid, int r, float a0, float a1, float xlo, float xhi,
                                       float cxx, float nmy, float scale) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    WRun w{0ull, 0ull};
    for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
        const bool inr = valid && x >= xlo && x <= xhi;
        const uint64_t q = q_of(ex2_approx(__fmaf_rn(x, cxx, nmy)), scale);
        w.acc += (inr && x > a1) ? q : 0ull;
        w.cnt += (inr && x <= a1 && x >= a0) ? 1u : 0u;
    });
    return w;
}
struct WCol { uint64_t acc, acc2; uint32_t kmn, kmx, kmn2, kmx2; };
// Collects the window [a0, a1], and the window [b0, b1] above it when b0 <=
// b1, into the buffer from slot0 (counter ctl->ncol, zero on entry); per
// thread, the mass above each window and the key range collected of each.
template <int DT>
__device__ __noinline__ WCol wpass_collect(const KParams& P, int tid, int r, float a0, float a1, float xlo, float xhi,
                                           float cxx, float nmy, float scale, uint32_t slot0, float b0, float b1) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    const int lane = tid & 31;
    WCol w{0ull, 0ull, 0xffffffffu, 0u, 0xffffffffu, 0u};
    for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
        const bool inr = valid && x >= xlo && x <= xhi;
        const bool inA = inr && x >= a0 && x <= a1;
        const bool inB = inr && x >= b0 && x <= b1;
        const bool in = inA || inB;
        const uint64_t qa = q_of(ex2_approx(__fmaf_rn(x, cxx, nmy)), scale);
        w.acc += (inr && x > a1) ? qa : 0ull;
        w.acc2 += (inr && x > b1) ? qa : 0ull;
        const uint32_t bal = __ballot_sync(0xffffffffu, in);
        if (bal) {
            const int lead = __ffs(bal) - 1;
            uint32_t b0 = 0u;
            if (lane == lead) b0 = atoms_add(&s.ctl->ncol, (uint32_t)__popc(bal));
            b0 = __shfl_sync(0xffffffffu, b0, lead);
            if (in) {
                const uint32_t k = fkey(ydiv(p, x));
                const uint32_t pos = slot0 + b0 + (uint32_t)__popc(bal & ((1u << lane) - 1u));
                if (pos < (uint32_t)CAND_CAP) { s.ckey[pos] = k; s.cid[pos] = (uint32_t)c; }
                if (inA) { w.kmn = min(w.kmn, k); w.kmx = max(w.kmx, k); }
                else { w.kmn2 = min(w.kmn2, k); w.kmx2 = max(w.kmx2, k); }
            }
        }
    });
    return w;
}

template <int DT>
__device__ __forceinline__ WLoc wlocate(const KParams& P, const Smem& s, const RowParams& p, int r, const RowGeom& g, int tid,
                        uint32_t rlo, uint32_t rhi, float ylo, float yhi, uint64_t target, float My, float scale,
                        uint32_t slot0, uint64_t target2) {
    WLoc W;
    Located& L = W.L;
    W.fallback = false;
    if (tid == 0) s.ctl->b_ok = 0u;
    L.ok = false; L.in_buffer = false; L.key = 0u; L.before = 0; L.at = 0; L.n_at = 0; L.total = 0;
    L.n0 = slot0; L.n1 = slot0;
    if (rlo > rhi) return W;
    const uint32_t room = slot0 < (uint32_t)CAND_CAP ? (uint32_t)CAND_CAP - slot0 : 0u;
    const uint32_t fit = room - room / 8u;   // margin for the edge slack and tie closure
    uint32_t* cnt = s.blo;                   // NW words (blo and bhi are contiguous)
    // region in x; below `cutoff` under the maximum a mass rounds to 0 at scale 2^S
    const float cutoff = (float)(P.mass_shift + 2) * 0.6931472f;
    // the region's top is its largest y (yhi), so the window stays finite
    const float xlo = x_lower(p, rlo), xhi = x_upper(p, min(rhi, fkey(yhi)));
    const float xpos = x_lower(p, fkey(fmaxf(ylo, My - cutoff)));
    float wl = fmaxf(xlo, xpos), wu = xhi;   // current window (nested, closed under equal y)
    if (!(wu >= wl)) return W;               // every mass in R rounds to 0: total 0
    const float cx = L2E / p.T;              // m(x) = 2^(x * cx + nmy), cx == L2E when T == 1
    const float nmy = -(My * L2E);
    const float cxx = p.temp_on ? cx : L2E;
    const double sc = (double)scale;
    const double T = (double)target;
    uint64_t above = 0;
    bool beyond = false, single = false;
    // second window (level 0 only): the draw's, for target2 < target
    bool b_try = false;
    float bl = 1.0f, bu = 0.0f;
    uint32_t bcount = 0u, acount = 0u;
    for (int d = 0;; ++d) {
        // level 0 spans the whole region: twice the bins when the candidate
        // buffer's free part holds them (the collection overwrites them later)
        const bool big = d == 0 && room >= (uint32_t)NW0 + 64u;
        const int nb = big ? NW0 : NW;
        uint32_t* cl = big ? s.ckey + slot0 : cnt;
        const float span = wu - wl;
        float inv = span > 0.0f ? (float)nb / span : 0.0f;
        if (!(inv < INFINITY)) inv = 0.0f;
        const double sx = 1e-6 * (double)span;
        for (int i = tid; i < nb; i += NCT) cl[i] = 0u;
        csync();
        uint64_t acc = 0;
        const float a0 = wl, a1 = wu, bi = inv;
        if (d == 0) {
            // nothing lies above level 0's range: counts only
            if (big) wpass_count<DT, NW0>(P, tid, r, a0, bi, xlo, xhi, slot0);
            else wpass_count<DT, NW>(P, tid, r, a0, bi, xlo, xhi, slot0);
        } else {
            acc = wpass_mass<DT>(P, tid, r, a0, a1, bi, xlo, xhi, cxx, nmy, scale);
        }
        csync();
        if (d > 0) above = cons_sum_u64(acc, s, tid);
        const WWin win = big ? wscan<NW0>(s, cl, wl, wu, inv, sx, p, My, sc, (double)above, T, tid)
                             : wscan<NW>(s, cl, wl, wu, inv, sx, p, My, sc, (double)above, T, tid);
        if (!win.any) { beyond = true; break; }
        const double w = inv > 0.0f ? 1.0 / (double)inv : 0.0;
        if (d == 0 && target2 < target) {
            const WWin w2 = big ? wscan<NW0>(s, cl, wl, wu, inv, sx, p, My, sc, 0.0, (double)target2, tid)
                                : wscan<NW>(s, cl, wl, wu, inv, sx, p, My, sc, 0.0, (double)target2, tid);
            if (w2.any && w > 0.0) {
                float l2 = wl, u2 = wu;
                if (w2.lo > 0) l2 = __double2float_rd((double)wl + (double)w2.lo * w - sx);
                if (w2.hi < nb - 1) u2 = __double2float_ru((double)wl + (double)(w2.hi + 1) * w + sx);
                bl = fmaxf(wl, x_lower(p, fkey(ydiv(p, l2))));
                bu = fminf(wu, x_upper(p, fkey(ydiv(p, u2))));
                bcount = w2.count;
                b_try = bu >= bl;
            }
        }
        acount = win.count;
        // the window's x-range, widened by the slack, closed under equal y
        float nl = wl, nu = wu;
        if (w > 0.0) {
            if (win.lo > 0) nl = __double2float_rd((double)wl + (double)win.lo * w - sx);
            if (win.hi < nb - 1) nu = __double2float_ru((double)wl + (double)(win.hi + 1) * w + sx);
        }
        nl = fmaxf(wl, x_lower(p, fkey(ydiv(p, nl))));
        nu = fminf(wu, x_upper(p, fkey(ydiv(p, nu))));
        const bool progress = nl > wl || nu < wu;
        wl = nl;
        wu = nu;
        if (win.count <= fit) break;
        // a window of one value (a run of ties longer than the free buffer)
        // cannot be split further, and need not be collected
        if (fkey(ydiv(p, wl)) == fkey(ydiv(p, wu))) { single = true; break; }
        if (d + 1 >= WDEPTH || !progress) {
            W.fallback = true;
            return W;
        }
    }
    if (single) {
        // exact mass above the run and its length; every element of the run
        // has the same y, hence the same mass
        const float a0 = wl, a1 = wu;
        const WRun wr = wpass_run<DT>(P, tid, r, a0, a1, xlo, xhi, cxx, nmy, scale);
        const uint64_t accA = wr.acc, cnt = wr.cnt;
        const uint64_t A = cons_sum_u64(accA, s, tid);
        const uint64_t n_at = cons_sum_u64(cnt, s, tid);
        const uint32_t key = fkey(ydiv(p, wl));
        const uint64_t q = q_of(efast(funkey(key), My), scale);
        if (target < A) { W.fallback = true; return W; }   // bracket violated: take the exact path
        if (n_at == 0 || target >= A + n_at * q) {
            L.total = region_mass<DT>(P, s, p, r, g, tid, rlo, rhi, My, scale);
            if (target < L.total) W.fallback = true;
            return W;
        }
        L.ok = true; L.in_buffer = false; L.key = key; L.before = A; L.at = n_at * q; L.n_at = (uint32_t)n_at;
        L.total = A + n_at * q;
        return W;
    }
    if (beyond) {
        // the target lies at or past the region's total mass
        L.total = region_mass<DT>(P, s, p, r, g, tid, rlo, rhi, My, scale);
        return W;
    }
    // ---- collect the window [wl, wu]; exact mass above it ----
    if (tid == 0) s.ctl->ncol = 0u;
    csync();
    const float a0 = wl, a1 = wu;
    // the draw's window rides along when it lies wholly above this one and
    // both fit the free buffer
    const bool use_b = b_try && bl > a1 && acount + bcount <= fit;
    const WCol wc = wpass_collect<DT>(P, tid, r, a0, a1, xlo, xhi, cxx, nmy, scale, slot0, use_b ? bl : 1.0f,
                                      use_b ? bu : 0.0f);
    uint32_t kmn = wc.kmn, kmx = wc.kmx;
    const uint64_t A = cons_sum_u64(wc.acc, s, tid);
    kmn = cons_min_u32(kmn, s, tid);
    kmx = cons_max_u32(kmx, s, tid);
    const uint32_t ncol = s.ctl->ncol;
    if (ncol > room) { W.fallback = true; return W; }
    const uint32_t n1 = slot0 + ncol;
    uint64_t wloc = 0, wloc2 = 0;
    for (uint32_t i = slot0 + tid; i < n1; i += NCT) {
        const uint32_t k = s.ckey[i];
        const uint64_t q = q_of(efast(funkey(k), My), scale);
        if (k <= kmx) wloc += q; else wloc2 += q;
    }
    const uint64_t Wm = cons_sum_u64(wloc, s, tid);
    if (use_b) {
        const uint64_t A2 = cons_sum_u64(wc.acc2, s, tid);
        const uint64_t W2 = cons_sum_u64(wloc2, s, tid);
        const uint32_t k2n = cons_min_u32(wc.kmn2, s, tid);
        const uint32_t k2x = cons_max_u32(wc.kmx2, s, tid);
        if (tid == 0 && W2 > 0 && k2n > kmx && k2n <= k2x) {
            s.ctl->b_ok = 1u; s.ctl->b_klo = k2n; s.ctl->b_khi = k2x; s.ctl->b_n1 = n1;
            s.ctl->b_above = A2; s.ctl->b_mass = W2;
        }
    }
    if (target < A) { W.fallback = true; return W; }   // bracket violated: take the exact path
    if (target >= A + Wm) {
        // past the window: only when the target is past the region's total
        L.total = region_mass<DT>(P, s, p, r, g, tid, rlo, rhi, My, scale);
        if (target < L.total) W.fallback = true;
        return W;
    }
    const SelOut so = block_select<true, false>(
        [&](auto&& f) {
            for (uint32_t i0 = slot0; i0 < n1; i0 += NCT) {
                const uint32_t i = i0 + tid;
                const uint32_t k = i < n1 ? s.ckey[i] : 0u;
                const bool v = i < n1 && k <= kmx;
                f(v, k, v ? q_of(efast(funkey(k), My), scale) : 0ull);
            }
        },
        target - A, kmn, varying_bits(kmn, kmx), s, tid);
    L.ok = so.ok; L.in_buffer = true; L.key = so.key; L.before = A + so.before; L.at = so.at; L.n_at = so.n_at;
    L.n0 = slot0; L.n1 = n1;
    L.total = A + Wm;   // mass at and above the window (the part below is not needed)
    if (!so.ok) W.fallback = true;
    return W;
}

// Cold entry points of the multi-pass paths. They take only the kernel
// parameters (grid constant), the row and scalars, and rebuild the shared
// memory carve, row parameters and geometry themselves: no struct of the
// streaming loop has its address taken, so it stays in registers.
template <int DT>
__device__ __noinline__ WLoc wlocate_cold(const KParams& P, int tid, int r, uint32_t rlo, uint32_t rhi, float ylo,
                                          float yhi, uint64_t target, float My, float scale, uint32_t slot0,
                                          uint64_t target2) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    return wlocate<DT>(P, s, p, r, g, tid, rlo, rhi, ylo, yhi, target, My, scale, slot0, target2);
}
template <int DT>
__device__ __noinline__ Located locate_cold(const KParams& P, int tid, int r, uint32_t rlo, uint32_t rhi, float ylo,
                                            float yhi, uint64_t target, float My, float scale, uint32_t slot0) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    return locate<DT>(P, s, p, r, g, tid, rlo, rhi, ylo, yhi, target, My, scale, slot0);
}
template <int DT>
__device__ __noinline__ uint64_t region_mass_cold(const KParams& P, int tid, int r, uint32_t rlo, uint32_t rhi,
                                                  float My, float scale) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    return region_mass<DT>(P, s, p, r, g, tid, rlo, rhi, My, scale);
}

template <int DT>
__device__ __forceinline__ Located locate_fast(const KParams& P, const Smem& s, const RowParams& p, int r, const RowGeom& g,
                               int tid, uint32_t rlo, uint32_t rhi, float ylo, float yhi, uint64_t target, float My,
                               float scale, uint32_t slot0, bool clamp, uint64_t target2 = ~0ull) {
    (void)p; (void)g;
    WLoc w = wlocate_cold<DT>(P, tid, r, rlo, rhi, ylo, yhi, target, My, scale, slot0, target2);
    // like locate(), a clamped call answers a target past the total with the last element
    if (clamp && !w.fallback && !w.L.ok && w.L.total > 0 && target >= w.L.total)
        w = wlocate_cold<DT>(P, tid, r, rlo, rhi, ylo, yhi, w.L.total - 1, My, scale, slot0, ~0ull);
    if (!w.fallback) return w.L;
    if (tid == 0) s.ctl->b_ok = 0u;   // the exact path reuses the buffer
    return locate_cold<DT>(P, tid, r, rlo, rhi, ylo, yhi, target, My, scale, slot0);
}

// j-th smallest column (0-based) among entries [i0, i1) with key k.
__device__ __forceinline__ uint32_t jth_id(const KParams& P, const Smem& s, int tid, uint32_t i0, uint32_t i1,
                                           uint32_t k, uint32_t n_at, uint64_t j) {
    if (n_at <= 1 || j == 0) {
        uint32_t best = 0xffffffffu;
        for (uint32_t i = i0 + tid; i < i1; i += NCT) if (s.ckey[i] == k) best = min(best, s.cid[i]);
        return cons_min_u32(best, s, tid);
    }
    const SelOut si = block_select<false, true>(
        [&](auto&& f) {
            for (uint32_t b = i0; b < i1; b += NCT) {
                const uint32_t i = b + tid;
                const bool v = i < i1 && s.ckey[i] == k;
                f(v, v ? s.cid[i] : 0u, 1ull);
            }
        },
        j, 0u, P.id_bits, s, tid);
    return si.key;
}
// j-th smallest column among the row's elements whose y-key is k (row pass).
template <int DT>
__device__ uint32_t jth_id_row(const KParams& P, const Smem& s, const RowParams& p, int r, const RowGeom& g, int tid,
                               uint32_t k, uint64_t j) {
    const SelOut si = block_select<false, true>(
        [&](auto&& f) {
            for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
                const bool v = valid && fkey(ydiv(p, x)) == k;
                f(v, (uint32_t)c, 1ull);
            });
        },
        j, 0u, P.id_bits, s, tid);
    return si.key;
}

// ---------------------------------------------------------------------------
// Producer warp (one elected lane): row queue + bulk copies into the ring
// ---------------------------------------------------------------------------
template <int DT>
__device__ void producer(const KParams& P, const Smem& s) {
    constexpr int ESZ = Elem<DT>::SIZE;
    constexpr int HEAVY = 1 << 30;   // queue entry flag: the row may be re-read after its stream
    volatile int* abort = &s.ctl->abort;
    const uint32_t ns = (uint32_t)P.nstage;
    const unsigned B = (unsigned)P.batch;
    uint32_t it = 0, k = 0, st = 0, ph = 0;
    int held[ROW_CLAIM];
    int nheld = 0, hpos = 0;
    const uint64_t pol_keep = l2_policy_evict_last();
    // next owned queue entry (row | HEAVY), -1 when the queue is exhausted
    auto fetch = [&]() -> int {
        while (hpos == nheld) {
            const unsigned v = atomicAdd(&P.ws->next_row, (unsigned)ROW_CLAIM);
            if (v >= 2u * B) return -1;
            bool hv[ROW_CLAIM];
#pragma unroll
            for (int i = 0; i < ROW_CLAIM; ++i) hv[i] = (v + i < 2u * B) && row_heavy(P, (int)((v + i) % B));
            nheld = 0; hpos = 0;
#pragma unroll
            for (int i = 0; i < ROW_CLAIM; ++i) {
                const unsigned u = v + (unsigned)i;
                if (u < 2u * B && (u < B) == hv[i] && row_wanted(P, (int)(u % B)))
                    held[nheld++] = (int)(u % B) | (hv[i] ? HEAVY : 0);
            }
        }
        return held[hpos++];
    };
    auto drain = [&]() {
        const uint32_t first = it > ns ? it - ns : 0u;
        for (uint32_t j = first; j < it; ++j) mbar_wait_for(&s.full[j % ns], (j / ns) & 1u, WAIT_LIMIT_NS);
    };
    auto mark = [&](int e) {
        if (e < 0) return;
        const int rr = e & (HEAVY - 1);
        P.out_ids[rr] = -1;
        if (P.out_status) P.out_status[rr] = FG_ROW_TIMEOUT;
    };
    auto give_up = [&](int e) {
        *abort = 1;
        mark(e);
        while (hpos < nheld) mark(held[hpos++]);   // claimed, never published
        drain();
    };
    uint32_t nrow = 0, served = 0;
    int e = fetch();
    while (true) {
        const uint32_t slot = k % RQ, rph = (k / RQ) & 1u;
        if (!mbar_wait(&s.rowempty[slot], rph ^ 1u, abort)) { give_up(e); return; }
        s.ctl->rowq[slot] = e < 0 ? -1 : (e & (HEAVY - 1));
        mbar_arrive(&s.rowfull[slot]);
        ++k;
        if (e < 0) return;
        const int rcur = e & (HEAVY - 1);
        // rows that may be re-read after the stream stay in L2 until the
        // consumers release them (sample_row returns them to normal priority)
        const bool keep = (e & HEAVY) != 0;
        const RowGeom g = row_geom<ESZ>(P, rcur);
        // the row's interior, tile by tile, through the ring
        auto stream = [&]() -> bool {
            for (int t = 0; t < g.ntiles; ++t, ++it) {
                if (!mbar_wait(&s.empty[st], ph ^ 1u, abort)) return false;
                const int64_t off = (int64_t)t * TILE_BYTES;
                const int64_t left = g.interior_bytes - off;
                const uint32_t bytes = (uint32_t)(left < TILE_BYTES ? left : TILE_BYTES);
                mbar_arrive_expect_tx(&s.full[st], bytes);
                if (keep) bulk_g2s_hint(s.ring + (int64_t)st * TILE_BYTES, g.interior + off, bytes, &s.full[st], pol_keep);
                else bulk_g2s(s.ring + (int64_t)st * TILE_BYTES, g.interior + off, bytes, &s.full[st]);
                if (++st == ns) { st = 0; ph ^= 1u; }
            }
            return true;
        };
        if (!stream()) { give_up(-1); return; }
        // Until the consumers release the row, stream it again for each pass
        // over it that they request (their multi-pass paths read the row
        // through the ring). The next row is claimed only after the release,
        // so no claimed row waits behind a long one while other CTAs run out
        // of rows.
        ++nrow;
        {
            volatile uint32_t* go = &s.ctl->go;
            volatile uint32_t* preq = &s.ctl->preq;
            uint64_t t0 = globaltimer_ns();
            while (*go < nrow) {
                if (*preq != served) {
                    ++served;
                    if (!stream()) { give_up(-1); return; }
                    t0 = globaltimer_ns();
                    continue;
                }
                if (*abort || globaltimer_ns() - t0 > WAIT_LIMIT_NS) { give_up(-1); return; }
                __nanosleep(64);
            }
        }
        e = fetch();
    }
}

// ---------------------------------------------------------------------------
// Consumer warps: one row
// ---------------------------------------------------------------------------
struct RingPos { uint32_t st, ph; };

// ---------------------------------------------------------------------------
// Sorted candidate set: the finish of a row whose decision lies inside the
// candidate buffer. The buffer's (y-key, column) pairs are sorted once, in
// place, into descending key order with ties in ascending column order (the
// draw order), so the K-th key, the top-p cut and the draw are positions in
// one prefix of the sorted array: the first position whose inclusive prefix
// mass exceeds a target. Same integer masses and the same comparisons as the
// radix selects they replace, hence the same token. The bitonic sort costs
// O(n log^2 n) against the selects' few O(n) passes with their fixed costs, so
// it serves small sets only (the top-k rows with small K).
// ---------------------------------------------------------------------------
constexpr uint32_t SORT_MAX = 512;
__device__ __noinline__ void sort_cands_desc(const KParams& P, int tid, uint32_t n) {
    const Smem s = carve(smem_base(), P);
    uint32_t N = 2;
    while (N < n) N <<= 1;
    for (uint32_t i = n + tid; i < N; i += NCT) { s.ckey[i] = 0u; s.cid[i] = 0xffffffffu; }
    csync();
    for (uint32_t k = 2; k <= N; k <<= 1) {
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
            for (uint32_t t = tid; t < N / 2; t += NCT) {
                const uint32_t i = ((t & ~(j - 1u)) << 1) | (t & (j - 1u));
                const uint32_t l = i + j;
                const uint32_t ki = s.ckey[i], kl = s.ckey[l];
                const uint32_t ii = s.cid[i], il = s.cid[l];
                const bool first = ki > kl || (ki == kl && ii < il);   // i precedes l in the draw order
                const bool desc = (i & k) == 0u;
                if (desc != first) { s.ckey[i] = kl; s.ckey[l] = ki; s.cid[i] = il; s.cid[l] = ii; }
            }
            csync();
        }
    }
}

// First position i in [0, lim) of the sorted buffer whose inclusive prefix
// mass exceeds T (T below the mass of [0, lim)); *incl = that prefix mass.
__device__ __noinline__ uint32_t sorted_crossing(const KParams& P, int tid, uint32_t lim, uint64_t T, float My,
                                                float scale, uint64_t* incl) {
    const Smem s = carve(smem_base(), P);
    const int lane = tid & 31, wid = tid >> 5;
    const uint32_t E = (lim + NCT - 1) / NCT;
    const uint32_t i0 = min(lim, (uint32_t)tid * E), i1 = min(lim, i0 + E);
    auto q = [&](uint32_t i) { return q_of(expf(funkey(s.ckey[i]) - My), scale); };
    uint64_t S = 0;
    for (uint32_t i = i0; i < i1; ++i) S += q(i);
    // exclusive prefix of the per-thread sums (threads in index order)
    uint64_t x = S;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t y = shfl_u64(x, (lane - o) & 31);
        if (lane >= o) x += y;
    }
    if (lane == 31) s.red64[wid] = x;
    csync();
    uint64_t base = x - S;
    for (int w = 0; w < NCW; ++w) if (w < wid) base += s.red64[w];
    if (tid == 0) { s.ctl->ncol = 0xffffffffu; }
    csync();
    if (base <= T && T < base + S) {
        uint64_t acc = base;
        for (uint32_t i = i0; i < i1; ++i) {
            acc += q(i);
            if (acc > T) { s.ctl->ncol = i; *reinterpret_cast<uint64_t*>(s.redd) = acc; break; }
        }
    }
    csync();
    const uint32_t r = s.ctl->ncol;
    *incl = *reinterpret_cast<const uint64_t*>(s.redd);
    csync();
    return r;
}

// ---------------------------------------------------------------------------
// After the stream: row statistics, the decision (greedy / sampling), outputs.
// ---------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void finish_row(const KParams& P, const Smem& s, const int tid, const int r, const RowParams& p,
                                        const RowGeom& g, const Stream& st, const bool aborted) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE, VEC = E::VEC;
    (void)ESZ;
    RowCtl* ctl = s.ctl;
    volatile int* abort = &ctl->abort;
    const float scale = __uint_as_float((uint32_t)(127 + P.mass_shift) << 23);  // 2^S
    // ---- row statistics ----
    const float M = cons_max_nan(st.tmax, s, tid);
    int status = ctl->status;
    const uint32_t n = st.base;
    // a top-k row whose filter (started from a sample of the row) kept fewer
    // than K elements runs its select over the whole row
    const bool cand_ok = st.cand && !aborted && (p.mode != MODE_TOPK || n >= (uint32_t)p.K);
    double Zq = 0.0;
    float My = M;
    float ymin = -INFINITY;
    if (p.zsum && !aborted && M == M && M > -INFINITY && M < INFINITY) {
        My = ydiv(p, M);
        double zc = 0.0;
        const double zsum = (double)st.z0 + (double)st.z1;
        if (zsum > 0.0) zc = zsum * exp2(-(double)st.nzmc - (double)M * (double)p.c);
        const double Zd = cons_sum_f64(zc, s, tid);
        Zq = Zd * exp((double)M / (double)p.T - (double)My) * (double)scale;
        ymin = ydiv(p, cons_min_f(st.tmin, s, tid));
    }
    // merge stage of the split path: the row's total mass from the shards'
    // partials (the union holds only their candidates), the key from which
    // the union is complete, and the shards' status words
    uint32_t thr_max = 0u;
    int shard_or = 0;
    bool split_redo = false;
    if (P.merge_g > 0) {
        // one lane of warp 0 per shard (merge_g <= 32)
        if (tid < 32) {
            double z = 0.0;
            uint32_t th = 0u, so = 0u;
            if (tid < P.merge_g) {
                const int64_t sj = (int64_t)r * P.merge_g + tid;
                th = __ldg(P.shard_thr + sj);
                so = (uint32_t)__ldg(P.shard_status + sj);
                const double my = __ldg(P.shard_mz + 2 * sj), zz = __ldg(P.shard_mz + 2 * sj + 1);
                if (zz > 0.0) z = zz * exp(my - (double)My);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
            th = __reduce_max_sync(0xffffffffu, th);
            so = __reduce_or_sync(0xffffffffu, so);
            if (tid == 0) { s.redd[0] = z; s.red32[0] = th; s.red32[1] = so; }
        }
        csync();
        const double zt = s.redd[0];
        thr_max = s.red32[0];
        shard_or = (int)s.red32[1];
        csync();
        if (p.zsum && Zq > 0.0) Zq = zt * (double)scale;
        // a shard whose columns are all -inf just has an empty set
        split_redo = (shard_or & (FG_ROW_ERROR_MASK & ~FG_ROW_ALL_MASKED)) != 0;
    }
    int64_t out_id = -1;
    bool cand_written = false;   // candidates mode: this row's set was written
    float* pr = P.out_probs ? P.out_probs + (int64_t)r * P.vocab : nullptr;

    if (aborted) {
        status |= FG_ROW_TIMEOUT;
    } else if (status & (FG_ROW_BAD_PARAM | FG_ROW_BAD_UNIFORM)) {
        out_id = -1;
    } else if (p.mode == MODE_GREEDY) {
        status |= FG_ROW_GREEDY;
        uint32_t best = 0xffffffffu;
        if (M != M) {
            for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) { if (valid && x != x) best = min(best, (uint32_t)c); });
            status |= FG_ROW_GENERAL_PATH;
        } else {
            if (st.bestv == M) best = st.bestc;
            if (st.imax == M && st.itile >= 0) {
                // first column of this thread's chunks in that tile holding M
                const int t = st.itile;
                const int64_t left = g.interior_bytes - (int64_t)t * TILE_BYTES;
                const int nch = (int)((left < TILE_BYTES ? left : TILE_BYTES) / 16);
                const int tcol0 = g.head + t * (TILE_BYTES / ESZ);
                for (int j = 0; j < CPT; ++j) {
                    const int ch = tid + j * NCT;
                    if (ch >= nch) break;
                    const uint4 v = __ldg(reinterpret_cast<const uint4*>(g.interior + (int64_t)t * TILE_BYTES) + ch);
                    const int c0 = tcol0 + ch * VEC;
                    const uint32_t hbits = p.pen ? hist_bits(s, P.nwords, c0, VEC) : 0u;
                    int found = -1;
#pragma unroll
                    for (int e = VEC - 1; e >= 0; --e)
                        if (!((hbits >> e) & 1u) && elem_get<DT>(v, e) == M) found = e;
                    if (found >= 0) { best = min(best, (uint32_t)(c0 + found)); break; }
                }
            }
        }
        best = cons_min_u32(best, s, tid);
        out_id = best;
        if (P.cand_vals != nullptr) {
            // candidates mode: the shard's first maximum (the merge takes the
            // first maximum over the shards' ones, in global-id order)
            float* cv = P.cand_vals + (int64_t)r * P.cand_max;
            int32_t* cg = P.cand_ids + (int64_t)r * P.cand_max;
            const bool any = best != 0xffffffffu;
            for (int i = tid; i < P.cand_max; i += NCT) {
                cv[i] = (i == 0 && any) ? M : -INFINITY;
                cg[i] = (i == 0 && any) ? (int32_t)(best + col_base(P, r)) : INT32_MAX;
            }
            if (tid == 0) {
                P.cand_count[r] = any ? 1 : 0;
                if (P.cand_mz != nullptr) {
                    P.cand_thr[r] = 0xffffffffu;
                    P.cand_mz[2 * (int64_t)r] = 0.0;
                    P.cand_mz[2 * (int64_t)r + 1] = 0.0;
                }
            }
            cand_written = true;
        }
        if (pr) for (int c = tid; c < P.vocab; c += NCT) pr[c] = (c == (int)best) ? 1.0f : 0.0f;
    } else if (M != M) {
        status |= FG_ROW_NAN;
    } else if (M == INFINITY) {
        status |= FG_ROW_POS_INF;
    } else if (M == -INFINITY) {
        status |= FG_ROW_ALL_MASKED;
    } else {
        // ================= sampling rows =================
        My = ydiv(p, M);
        const uint32_t hiY = fkey(My);
        if (ymin < My - 64.0f || !(ymin == ymin)) ymin = My - 64.0f;   // masses below are 0 at 2^-S
        // candidate set C = {y >= y(xmin)} (complete); empty when the filter overflowed
        uint32_t nC = cand_ok ? n : 0u;
        const uint32_t loY = cand_ok ? fkey(ydiv(p, ctl->xmin)) : 0xffffffffu;
        if (nC > 0) {
            for (uint32_t i = tid; i < nC; i += NCT) s.ckey[i] = fkey(ydiv(p, funkey(s.ckey[i])));
            csync();
        }
        const uint32_t cLo = min(loY, hiY);
        const int remC = varying_bits(cLo, hiY);
        auto qC = [&](uint32_t yk) { return q_of(expf(funkey(yk) - My), scale); };   // exact masses in C
        // the sampling rows' candidate sets are sorted into the draw order
        const bool sorted = nC > 0 && nC <= SORT_MAX && P.cand_vals == nullptr;
        if (sorted) sort_cands_desc(P, tid, nC);
        // top-k threshold (on C, or over the whole row when C cannot hold it)
        uint32_t ykK = 0u;
        if (p.mode == MODE_TOPK) {
            if (cand_ok && sorted) {
                ykK = s.ckey[p.K - 1];   // nC >= K
            } else if (cand_ok) {
                const SelOut so = block_select<true, true>(
                    [&](auto&& f) {
                        for (uint32_t i0 = 0; i0 < nC; i0 += NCT) {
                            const uint32_t i = i0 + tid;
                            f(i < nC, i < nC ? s.ckey[i] : 0u, 1ull);
                        }
                    },
                    (uint64_t)(p.K - 1), cLo, remC, s, tid);
                ykK = so.ok ? so.key : 0u;
            } else {
                const SelOut so = block_select<true, true>(
                    [&](auto&& f) {
                        for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
                            f(valid && x == x, fkey(ydiv(p, x)), 1ull);
                        });
                    },
                    (uint64_t)(p.K - 1), 0u, 32, s, tid);
                ykK = so.ok ? so.key : 0u;
                nC = 0;
            }
        }
        auto keepk = [&](uint32_t yk) { return p.mode != MODE_TOPK || yk >= ykK; };
        if (P.cand_vals != nullptr && P.cand_mz != nullptr) {
            // shard stage of the split path: the shard's top-k set (top-k
            // rows) or its top cand_max values (other rows), in column order,
            // with the key from which the output is complete and the shard's
            // mass partial
            uint32_t klo_out = 0u, thr = 0u;
            bool trunc = !cand_ok;
            if (cand_ok && p.mode == MODE_TOPK) {
                klo_out = ykK; thr = ykK;
            } else if (cand_ok && nC > (uint32_t)P.cand_max) {
                const SelOut so = block_select<true, true>(
                    [&](auto&& f) {
                        for (uint32_t i0 = 0; i0 < nC; i0 += NCT) {
                            const uint32_t i = i0 + tid;
                            f(i < nC, i < nC ? s.ckey[i] : 0u, 1ull);
                        }
                    },
                    (uint64_t)(P.cand_max - 1), cLo, remC, s, tid);
                if (!so.ok || so.key == 0xffffffffu) trunc = true;
                klo_out = so.key + 1u; thr = klo_out;
            } else if (cand_ok) {
                klo_out = 0u; thr = loY;
            }
            if (tid == 0) ctl->ncol = 0u;
            csync();
            if (!trunc) {
                for (uint32_t i = tid; i < nC; i += NCT) {
                    if (s.ckey[i] < klo_out) continue;
                    const uint32_t pos = atoms_add(&ctl->ncol, 1u);
                    if (pos < (uint32_t)P.cand_max) { s.blo[pos] = s.ckey[i]; s.bhi[pos] = s.cid[i]; }
                }
            }
            csync();
            const uint32_t cnt = ctl->ncol;
            if (trunc || cnt > (uint32_t)P.cand_max) status |= FG_ROW_CAND_TRUNC;
            const uint32_t w = min(cnt, (uint32_t)P.cand_max);
            float* cv = P.cand_vals + (int64_t)r * P.cand_max;
            int32_t* cg = P.cand_ids + (int64_t)r * P.cand_max;
            const int64_t cb = col_base(P, r);
            // position = rank by column among the output (columns are distinct)
            for (uint32_t i = tid; i < w; i += NCT) {
                const uint32_t ci = s.bhi[i];
                uint32_t rank = 0;
                for (uint32_t j = 0; j < w; ++j) rank += s.bhi[j] < ci ? 1u : 0u;
                cv[rank] = funkey(s.blo[i]);
                cg[rank] = (int32_t)(ci + cb);
            }
            for (uint32_t i = w + tid; i < (uint32_t)P.cand_max; i += NCT) { cv[i] = -INFINITY; cg[i] = INT32_MAX; }
            cand_written = true;
            if (tid == 0) {
                P.cand_count[r] = (int32_t)w;
                P.cand_thr[r] = thr;
                P.cand_mz[2 * (int64_t)r] = (double)My;
                P.cand_mz[2 * (int64_t)r + 1] = Zq / (double)scale;
            }
        } else if (P.cand_vals != nullptr) {
            // candidates mode (a vocabulary shard): the row's top-k set, ties
            // included, as (y, global id); the draw happens after the merge
            if (p.mode != MODE_TOPK) {
                status |= FG_ROW_BAD_PARAM;   // top-k off needs the whole distribution
            } else {
                if (tid == 0) ctl->ncol = 0u;
                csync();
                float* cv = P.cand_vals + (int64_t)r * P.cand_max;
                int32_t* cg = P.cand_ids + (int64_t)r * P.cand_max;
                auto put = [&](uint32_t yk, uint32_t col) {
                    const uint32_t pos = atoms_add(&ctl->ncol, 1u);
                    if (pos < (uint32_t)P.cand_max) { cv[pos] = funkey(yk); cg[pos] = (int32_t)(col + col_base(P, r)); }
                };
                if (nC > 0) {
                    for (uint32_t i = tid; i < nC; i += NCT) if (s.ckey[i] >= ykK) put(s.ckey[i], s.cid[i]);
                } else {
                    for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
                        if (!valid || !(x == x)) return;
                        const uint32_t yk = fkey(ydiv(p, x));
                        if (yk >= ykK) put(yk, (uint32_t)c);
                    });
                }
                csync();
                const uint32_t cnt = ctl->ncol;
                if (cnt > (uint32_t)P.cand_max) status |= FG_ROW_CAND_TRUNC;
                const uint32_t w = min(cnt, (uint32_t)P.cand_max);
                for (uint32_t i = w + tid; i < (uint32_t)P.cand_max; i += NCT) { cv[i] = -INFINITY; cg[i] = INT32_MAX; }
                if (tid == 0) P.cand_count[r] = (int32_t)w;
            }
        } else {
        uint64_t loc = 0, nloc = 0;
        for (uint32_t i = tid; i < nC; i += NCT) if (keepk(s.ckey[i])) { loc += qC(s.ckey[i]); ++nloc; }
        const uint64_t AC = cons_sum_u64(loc, s, tid);   // exact mass of the kept part of C
        // the kept part of a sorted C is its prefix [0, nk)
        const uint32_t nk = sorted ? (uint32_t)cons_sum_u64(nloc, s, tid) : 0u;

        // region R below C (whole row when C is empty), restricted to y >= T_K for top-k
        const uint32_t rlo = (p.mode == MODE_TOPK) ? ykK : KEY_NEG_INF;
        const uint32_t rhi = nC > 0 ? loY - 1u : 0xffffffffu;
        const float yRlo = (p.mode == MODE_TOPK) ? fmaxf(funkey(ykK), My - 64.0f) : ymin;
        const float yRhi = nC > 0 ? funkey(loY - 1u) : My;
        bool cut = false, cut_in_R = false;
        uint32_t tstar = 0u, id_cut = 0xffffffffu;
        uint32_t dkey = 0u;   // y-key of the drawn element when drawn from C
        uint64_t Qf = 0, m_t = 0, n_t = 0;
        if (p.use_p) {
            double Qn;
            if (p.mode == MODE_TOPK && cand_ok) Qn = (double)AC;
            else if (p.mode == MODE_TOPK) {
                Qn = (double)region_mass_cold<DT>(P, tid, r, rlo, rhi, My, scale);
            } else Qn = Zq;
            const double Pd = (double)p.top_p * Qn;
            const uint64_t Pt = (uint64_t)floor(Pd);
            cut = true;
            if ((double)AC > Pd && nC > 0 && sorted) {
                uint64_t incl = 0;
                const uint32_t ic = min(sorted_crossing(P, tid, nk, Pt, My, scale, &incl), nk - 1u);
                tstar = s.ckey[ic];
                // the run of entries with key tstar around ic (ties at the cut)
                uint32_t a = 0xffffffffu, b = 0u;
                for (uint32_t i = tid; i < nk; i += NCT)
                    if (s.ckey[i] == tstar) { a = min(a, i); b = max(b, i + 1u); }
                a = cons_min_u32(a, s, tid);
                b = cons_max_u32(b, s, tid);
                n_t = b - a;
                m_t = ic - a + 1u;
                Qf = incl;
            } else if ((double)AC > Pd && nC > 0) {
                const SelOut so = block_select<true, false>(
                    [&](auto&& f) {
                        for (uint32_t i0 = 0; i0 < nC; i0 += NCT) {
                            const uint32_t i = i0 + tid;
                            const uint32_t yk = i < nC ? s.ckey[i] : 0u;
                            const bool v = i < nC && keepk(yk);
                            f(v, yk, v ? qC(yk) : 0ull);
                        }
                    },
                    Pt, cLo, remC, s, tid);
                tstar = so.key;
                const uint64_t qt = so.n_at ? so.at / so.n_at : 0;
                m_t = so.n_at; n_t = so.n_at;
                if (qt > 0) { const uint64_t mm = (Pt - so.before) / qt + 1; if (mm < m_t) m_t = mm; }
                Qf = so.before + m_t * qt;
            } else {
                status |= FG_ROW_GENERAL_PATH;
                const uint64_t tr = Pt >= AC ? Pt - AC : 0ull;
                // the draw's target, predicted from Pt (the final Qf exceeds Pt by
                // less than one element's mass), so its window can be collected
                // in the same pass as the cut's
                uint64_t t2p = ~0ull;
                {
                    const uint64_t tg = (uint64_t)floor((double)p.u * (double)Pt);
                    if (tg >= AC && tg - AC < tr) t2p = tg - AC;
                }
                const Located L = locate_fast<DT>(P, s, p, r, g, tid, rlo, rhi, yRlo, yRhi, tr, My, scale, nC, false, t2p);
                if (!L.ok || tr >= L.total) {
                    cut = false;               // the cut lies below every element: keep all
                    Qf = AC + L.total;
                } else {
                    cut_in_R = true;
                    tstar = L.key;
                    const uint64_t qt = L.n_at ? L.at / L.n_at : 0;
                    m_t = L.n_at; n_t = L.n_at;
                    if (qt > 0) { const uint64_t mm = (tr - L.before) / qt + 1; if (mm < m_t) m_t = mm; }
                    Qf = AC + L.before + m_t * qt;
                }
            }
        } else {
            if (p.mode == MODE_TOPK && cand_ok) Qf = AC;
            else if (p.mode == MODE_TOPK) {
                Qf = region_mass_cold<DT>(P, tid, r, rlo, rhi, My, scale);
            } else Qf = (uint64_t)Zq;   // unfiltered: every token kept
        }
        // ---- inverse-CDF draw in descending-probability order ----
        if (Qf > 0) {
            uint64_t target = (uint64_t)floor((double)p.u * (double)Qf);
            if (target >= Qf) target = Qf - 1;
            if (target < AC && nC > 0 && sorted) {
                // kept entries within the cut form a prefix of the sorted buffer
                uint32_t lim = nk;
                if (cut && !cut_in_R) {
                    lim = 0u;
                    for (uint32_t i = tid; i < nk; i += NCT) if (s.ckey[i] >= tstar) lim = max(lim, i + 1u);
                    lim = cons_max_u32(lim, s, tid);
                    // only the first m_t entries of the tie run at tstar are kept
                    lim = (uint32_t)((uint64_t)lim - n_t + m_t);
                }
                uint64_t incl = 0;
                const uint32_t id = sorted_crossing(P, tid, lim, target, My, scale, &incl);
                if (id < lim) { out_id = s.cid[id]; dkey = s.ckey[id]; }
            } else if (target < AC && nC > 0) {
                const SelOut sd = block_select<true, false>(
                    [&](auto&& f) {
                        for (uint32_t i0 = 0; i0 < nC; i0 += NCT) {
                            const uint32_t i = i0 + tid;
                            const uint32_t yk = i < nC ? s.ckey[i] : 0u;
                            const bool v = i < nC && keepk(yk) && (!cut || cut_in_R || yk >= tstar);
                            f(v, yk, v ? qC(yk) : 0ull);
                        }
                    },
                    target, cLo, remC, s, tid);
                if (sd.ok) {
                    const uint64_t qd = sd.n_at ? sd.at / sd.n_at : 0;
                    uint64_t j = qd ? (target - sd.before) / qd : 0;
                    if (j >= sd.n_at) j = sd.n_at ? sd.n_at - 1 : 0;
                    out_id = jth_id(P, s, tid, 0u, nC, sd.key, sd.n_at, j);
                    dkey = sd.key;
                }
            } else {
                status |= FG_ROW_GENERAL_PATH;
                const uint64_t t2 = target - (nC > 0 ? AC : 0ull);
                bool drawn = false;
                if (cut_in_R && ctl->b_ok) {
                    const uint32_t bk0 = ctl->b_klo, bk1 = ctl->b_khi, bn1 = ctl->b_n1;
                    const uint64_t bA = ctl->b_above, bW = ctl->b_mass;
                    if (t2 >= bA && t2 - bA < bW) {
                        // inside the window collected with the cut's
                        const SelOut sb = block_select<true, false>(
                            [&](auto&& f) {
                                for (uint32_t i0 = nC; i0 < bn1; i0 += NCT) {
                                    const uint32_t i = i0 + tid;
                                    const uint32_t k = i < bn1 ? s.ckey[i] : 0u;
                                    const bool v = i < bn1 && k >= bk0 && k <= bk1;
                                    f(v, k, v ? q_of(efast(funkey(k), My), scale) : 0ull);
                                }
                            },
                            t2 - bA, bk0, varying_bits(bk0, bk1), s, tid);
                        if (sb.ok) {
                            const uint64_t qd = sb.n_at ? sb.at / sb.n_at : 0;
                            uint64_t j = qd ? (t2 - bA - sb.before) / qd : 0;
                            if (j >= sb.n_at) j = sb.n_at ? sb.n_at - 1 : 0;
                            out_id = jth_id(P, s, tid, nC, bn1, sb.key, sb.n_at, j);
                            dkey = sb.key;
                            drawn = true;
                        }
                    }
                }
                if (!drawn) {
                const uint32_t rlo2 = cut_in_R ? tstar : rlo;
                const float ylo2 = cut_in_R ? fmaxf(funkey(tstar), My - 64.0f) : yRlo;
                const Located L = locate_fast<DT>(P, s, p, r, g, tid, rlo2, rhi, ylo2, yRhi, t2, My, scale, nC, true);
                if (L.ok) {
                    const uint64_t qd = L.n_at ? L.at / L.n_at : 0;
                    uint64_t j = qd ? (t2 - L.before) / qd : 0;
                    if (j >= L.n_at) j = L.n_at ? L.n_at - 1 : 0;
                    out_id = L.in_buffer ? jth_id(P, s, tid, L.n0, L.n1, L.key, L.n_at, j)
                                         : jth_id_row<DT>(P, s, p, r, g, tid, L.key, j);
                }
                }   // !drawn
            }
        }
        // merge stage: exact only when the decision lies in the union's
        // complete part and inside the merge's candidate set
        if (P.merge_g > 0 && p.mode != MODE_TOPK) {
            if ((status & FG_ROW_GENERAL_PATH) || (cut && !cut_in_R && tstar < thr_max) || dkey < thr_max)
                split_redo = true;
        }
        if (out_id < 0 && !(status & FG_ROW_ERROR_MASK)) status |= FG_ROW_ALL_MASKED;
        // ---- kept-set probabilities (debug / oracle mode) ----
        if (pr && out_id >= 0) {
            // ties at the cut: the first m_t by ascending id are kept
            if (cut && m_t < n_t) {
                if (cut_in_R) {
                    id_cut = jth_id_row<DT>(P, s, p, r, g, tid, tstar, m_t - 1);
                } else {
                    const SelOut si = block_select<false, true>(
                        [&](auto&& f) {
                            for (uint32_t i0 = 0; i0 < nC; i0 += NCT) {
                                const uint32_t i = i0 + tid;
                                const bool v = i < nC && s.ckey[i] == tstar;
                                f(v, v ? s.cid[i] : 0u, 1ull);
                            }
                        },
                        m_t - 1, 0u, P.id_bits, s, tid);
                    id_cut = si.key;
                }
            }
            const double inv = 1.0 / (double)Qf;
            auto kept = [&](uint32_t yk, uint32_t c) {
                if (!keepk(yk)) return false;
                if (!cut) return true;
                if (yk > tstar) return true;
                if (yk < tstar) return false;
                return c <= id_cut;
            };
            for_row<DT>(P, s, p, r, g, tid, [&](bool valid, int c, float x) {
                if (!valid) return;
                const float y = ydiv(p, x);
                const uint32_t yk = fkey(y);
                float val = 0.0f;
                if (kept(yk, (uint32_t)c)) {
                    const bool inC = nC > 0 && yk >= loY;
                    const float e = inC ? expf(y - My) : efast(y, My);
                    val = (float)((double)q_of(e, scale) * inv);
                }
                pr[c] = val;
            });
        }
        }   // end of the sampling decision (not run in candidates mode)
    }
    if (pr && out_id < 0) for (int c = tid; c < P.vocab; c += NCT) pr[c] = 0.0f;
    if (P.cand_mz != nullptr && !cand_written) {
        // shard stage, no set written above (a row error): an empty set,
        // complete when the shard's columns are all -inf
        float* cv = P.cand_vals + (int64_t)r * P.cand_max;
        int32_t* cg = P.cand_ids + (int64_t)r * P.cand_max;
        for (int i = tid; i < P.cand_max; i += NCT) { cv[i] = -INFINITY; cg[i] = INT32_MAX; }
        if (tid == 0) {
            P.cand_count[r] = 0;
            P.cand_thr[r] = (status & FG_ROW_ERROR_MASK) == FG_ROW_ALL_MASKED ? 0u : 0xffffffffu;
            P.cand_mz[2 * (int64_t)r] = 0.0;
            P.cand_mz[2 * (int64_t)r + 1] = 0.0;
        }
    }
    if (tid == 0) {
        if (P.merge_g > 0) {
            // an error of the union itself (say, every shard's set empty after
            // a run of ties) is not the row's: the row is sampled whole
            if (status & FG_ROW_ERROR_MASK) split_redo = true;
            if (split_redo) { status |= FG_ROW_SPLIT_REDO; out_id = -1; }
            P.out_ids[r] = (out_id >= 0) ? (int64_t)__ldg(P.id_map + (int64_t)r * P.vocab + out_id) : -1;
            if (P.out_status) P.out_status[r] = status;
            if (P.final_status && !split_redo) P.final_status[r] = status;
        } else {
            P.out_ids[r] = (out_id >= 0) ? out_id + col_base(P, r) : -1;
            if (P.out_status) P.out_status[r] = status;
        }
    }
    csync();
    if (aborted && tid == 0) *abort = 1;
}

// Starting threshold of the candidate filter from the first tile (cold: once
// per row). Takes the thread's two chunks by value.
template <int DT>
__device__ __forceinline__ void tau0_cold(const KParams& P, int tid, int r, uint4 v0, uint4 v1, float m) {
    static_assert(CPT == 2, "tau0_cold takes CPT chunks by value");
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    RowCtl* ctl = s.ctl;
    constexpr int VEC = Elem<DT>::VEC;
    const uint4 v[CPT] = {v0, v1};
    // starting threshold from the first tile: the K-th largest of
    // disjoint group maxima (thread maxima for K <= NCT/2, chunk
    // maxima for K <= NCT, elements otherwise) of the tile. With K the
    // tile's share of the row's candidate target (1.5x, plus 8) rather than
    // the target itself, the filter passes about 1.5 target's worth of the
    // row on rows whose values are spread evenly along it, instead of every
    // tile's top K. The end of the row checks that the filter kept enough:
    // at least the row's top_k for top-k rows, enough mass for the nucleus
    // otherwise; a row that fails takes the whole-row path.
    float cm[CPT];
#pragma unroll
    for (int j = 0; j < CPT; ++j) cm[j] = chunk_max1<DT>(v[j]);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    const int64_t n0 = (g.interior_bytes < TILE_BYTES ? g.interior_bytes : TILE_BYTES) / Elem<DT>::SIZE;
    const int share = (int)ceilf(1.5f * (float)p.K * (float)n0 / (float)P.vocab) + 8;
    const int K = max(1, min(p.K, share));
    // key range of the values the select will see
    float lo_v = INFINITY;
    if (K <= NCT / 2) lo_v = m;
    else if (K <= NCT) { for (int j = 0; j < CPT; ++j) lo_v = fminf(lo_v, cm[j]); }
    else lo_v = chunks_min<DT>(v);
    // keys of the tile's raw values: 16-bit keys for the 16-bit dtypes
    auto kx = [&](float x) { return DT == FG_DTYPE_F32 ? fkey(x) : key16_of(fkey(x), DT); };
    uint32_t klo = (lo_v == lo_v && lo_v > -INFINITY) ? kx(lo_v) : 0xffffffffu;
    uint32_t khi = (m == m && m > -INFINITY) ? kx(m) : 0u;
    cons_minmax_u32(klo, khi, s, tid);
    const int kbits = DT == FG_DTYPE_F32 ? 32 : 16;
    const SelOut so = block_select<true, true>(
        [&](auto&& f) {
            if (K <= NCT / 2) {
                f(m == m && m > -INFINITY, m == m ? kx(m) : 0u, 1ull);
            } else if (K <= NCT) {
#pragma unroll
                for (int j = 0; j < CPT; ++j) f(cm[j] == cm[j] && cm[j] > -INFINITY, cm[j] == cm[j] ? kx(cm[j]) : 0u, 1ull);
            } else {
#pragma unroll
                for (int j = 0; j < CPT; ++j)
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        const float x = elem_get<DT>(v[j], e);
                        f(x == x && x > -INFINITY, x == x ? kx(x) : 0u, 1ull);
                    }
            }
        },
        (uint64_t)(K - 1), klo <= khi ? klo : 0u, klo <= khi ? varying_bits(klo, khi) : kbits, s, tid);
    if (so.ok && tid == 0) {
        const float xm = xmin_for(p, funkey(DT == FG_DTYPE_F32 ? so.key : key_from16(so.key, DT)));
        if (xm > ctl->xmin) ctl->xmin = xm;
    }
    csync();
}

__device__ __forceinline__ void history_prologue_cold(const KParams& P, int tid, int r) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    history_prologue(P, s, p, r, tid);
}

template <int DT>
__device__ __forceinline__ void finish_row_cold(const KParams& P, int tid, int r, float tmax, float tmin, float z0,
                                             float z1, float nzmc, bool cand, uint32_t base, float imax, int itile,
                                             float bestv, uint32_t bestc, bool aborted) {
    const Smem s = carve(smem_base(), P);
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    Stream st;
    st.tmax = tmax; st.tmin = tmin; st.z0 = z0; st.z1 = z1; st.nzmc = nzmc; st.zm = 0.0f; st.xmin = 0.0f;
    st.cand = cand; st.base = base; st.imax = imax; st.itile = itile; st.bestv = bestv; st.bestc = bestc;
    st.win = 0u; st.khi = 0u; st.klo = 0u;
    finish_row<DT>(P, s, tid, r, p, g, st, aborted);
}

// The streamed interior of one row: every tile of the ring through the
// history mask, max, sum-exp and candidate filter. Kept out of line, with only
// its own state live, so that the loop has the whole register budget; the
// stream state and ring position are copied in and written back once.
// Window schedule of the candidate filter within a row.
struct TileCtx {
    int last_chk, next_chk;   // tile of the last window end, tile of the next
    int span;                 // tiles in the window that just ended
    uint64_t rate2;           // twice the appends of that window
    uint32_t kcap;            // compact once the buffer holds more than this: the
                              // threshold then follows the K-th largest so far
};

// One streamed tile: history mask, max, sum-exp, candidate filter, window
// end. Returns true when a compaction is due (run by the caller, outside the
// streaming loop). FIRST: tile 0, which also sets the starting threshold.
template <int DT, bool FIRST>
__device__ __forceinline__ bool process_tile(const KParams& P, const RowParams& p, const RowGeom& g, const int tid,
                                             const int r, const int t, RingPos& rp, Stream& st, const uint32_t U,
                                             TileCtx& tc) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE, VEC = E::VEC;
    constexpr uint32_t O_ABORT = (uint32_t)offsetof(RowCtl, abort);
    constexpr uint32_t O_XMIN = (uint32_t)offsetof(RowCtl, xmin);
    constexpr uint32_t O_WCNT = (uint32_t)offsetof(RowCtl, wcnt);
    constexpr uint32_t O_OVF = (uint32_t)offsetof(RowCtl, ovf);
    const int lane = tid & 31;
    const uint32_t ns = (uint32_t)P.nstage;
    // shared-window addresses: symbol + grid-constant offsets, nothing held
    const uint32_t sb = smem_base32();
    const uint32_t a_ctl = sb + (uint32_t)P.off_ctl;
    const bool ok = mbar_wait_a(sb + 8u * rp.st, rp.ph, a_ctl + O_ABORT);
    if (!ok) sts_u32(a_ctl + O_ABORT, 1u);
    const uint32_t tile = sb + (uint32_t)P.off_ring + rp.st * (uint32_t)TILE_BYTES;
    const int64_t left = g.interior_bytes - (int64_t)t * TILE_BYTES;
    const int nch = ok ? (int)((left < TILE_BYTES ? left : TILE_BYTES) / 16) : 0;
    const int tcol0 = g.head + t * (TILE_BYTES / ESZ);
    uint4 v[CPT];
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
        const int ch = tid + j * NCT;
        if (ch < nch) v[j] = lds_v4(tile + (uint32_t)ch * 16u);
        else v[j] = make_uint4(Neg<DT>::W, Neg<DT>::W, Neg<DT>::W, Neg<DT>::W);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_a(sb + 8u * (ns + rp.st));   // the stage now lives in registers
    if (++rp.st == ns) { rp.st = 0; rp.ph ^= 1u; }
    uint32_t hb[CPT];
#pragma unroll
    for (int j = 0; j < CPT; ++j) hb[j] = 0u;
    if (p.pen) {
        const uint32_t bm = sb + (uint32_t)P.off_bitmap;
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            const int ch = tid + j * NCT;
            if (ch < nch) {
                const int c0 = tcol0 + ch * VEC;
                const int w = c0 >> 5, b = c0 & 31;
                const uint32_t lo = lds_u32(bm + 4u * (uint32_t)w);
                const uint32_t hi = (b + VEC > 32 && w + 1 < P.nwords) ? lds_u32(bm + 4u * (uint32_t)(w + 1)) : 0u;
                uint32_t bits = __funnelshift_r(lo, hi, b) & ((1u << VEC) - 1u);
                hb[j] = bits;
                while (bits) {
                    const int e = __ffs(bits) - 1;
                    bits &= bits - 1;
                    // rank of the column among the row's history columns
                    const uint32_t c = (uint32_t)(c0 + e), cw = c >> 5;
                    uint32_t rk = lds_u16(sb + (uint32_t)P.off_prefix + 2u * (cw >> 1)) +
                                  __popc(lds_u32(bm + 4u * cw) & ((1u << (c & 31)) - 1u));
                    if (cw & 1u) rk += __popc(lds_u32(bm + 4u * (cw - 1u)));
                    if (rk < U) sts_u32(sb + (uint32_t)P.off_sval + 4u * rk, __float_as_uint(elem_get<DT>(v[j], e)));
                    elem_mask<DT>(v[j], e);
                }
            }
        }
    }
    const float m = chunks_max<DT>(v);
    st.tmax = fmax_nan(st.tmax, m);
    if (p.mode == MODE_GREEDY && m > st.imax) { st.imax = m; st.itile = t; }
    if (p.zsum) {
        st.tmin = fminf(st.tmin, chunks_min<DT>(v));
        if (m > st.zm) {
            const float nn = -(m * p.c);
            const float f = ex2_approx(nn - st.nzmc);
            st.z0 *= f; st.z1 *= f;
            st.zm = m; st.nzmc = nn;
        }
        chunks_sumexp<DT>(v, p.c, st.nzmc, st.z0, st.z1);
    }
    if (st.cand) {
        if constexpr (FIRST) {
            tau0_cold<DT>(P, tid, r, v[0], v[1], m);
            st.xmin = __uint_as_float(lds_u32(a_ctl + O_XMIN));
        }
        uint32_t pick = 0;
        if (m >= st.xmin) {
            const uint32_t x2 = xmin_pair<DT>(st.xmin);
#pragma unroll
            for (int j = 0; j < CPT; ++j) {
                const int ch = tid + j * NCT;
                if (ch < nch) pick |= (chunk_ge<DT>(v[j], st.xmin, x2) & ~hb[j]) << (j * VEC);
            }
        }
        while (pick) {
            const int i = __ffs(pick) - 1;
            pick &= pick - 1;
            const int j = i / VEC, e = i % VEC;
            uint4 vv = v[0];
#pragma unroll
            for (int jj = 1; jj < CPT; ++jj) if (jj == j) vv = v[jj];
            const uint32_t key = fkey(elem_get<DT>(vv, e));
            const uint32_t col = (uint32_t)(tcol0 + (tid + j * NCT) * VEC + e);
            // append (no warp collectives: 32-bit shared atomics on one
            // counter are combined by the hardware)
            const uint32_t slot = st.win % 3u;
            const uint32_t pos = st.base + atoms_add_u32(a_ctl + O_WCNT + 4u * slot, 1u);
            if (pos < (uint32_t)CAND_CAP) {
                sts_u32(sb + (uint32_t)P.off_ckey + 4u * pos, key);
                sts_u32(sb + (uint32_t)P.off_cid + 4u * pos, col);
            } else {
                sts_u32(a_ctl + O_OVF + 4u * slot, 1u);
            }
            st.khi = max(st.khi, key);
            st.klo = min(st.klo, key);
        }
        // windows end where the previous check scheduled them (appends per
        // tile fall off as 1/t, so windows widen along the row), and at the
        // last tile; appends are bounds checked, an overflow sends the row
        // to the multi-pass path
        if (t == tc.next_chk || t == g.ntiles - 1) {
            const bool need = window_end(a_ctl, tid, st, (uint32_t)HWM, tc.kcap, tc.rate2);
            tc.span = t - tc.last_chk;
            tc.last_chk = t;
            if (need) return true;   // the caller compacts, then schedules the next window
            tc.next_chk = t + window_span(st.base, tc.rate2, tc.span, span_max_at(t));
        }
    }
    return false;
}

// Compaction after a window end (outside the streaming loop), then the next
// window's schedule.
__device__ __forceinline__ void compact_window(const KParams& P, const int tid, const int r, const int t, Stream& st,
                                               TileCtx& tc, int dt16) {
    const uint32_t a_ctl = smem_base32() + (uint32_t)P.off_ctl;
    const uint32_t n = compact_cold(P, tid, r, st.base, st.klo, st.khi, dt16);
    st.xmin = __uint_as_float(lds_u32(a_ctl + (uint32_t)offsetof(RowCtl, xmin)));
    st.klo = max(st.klo, fkey(st.xmin));
    st.base = n;
    if (n > (uint32_t)HWM) st.cand = false;
    if (2u * n > tc.kcap) tc.kcap = 2u * n;   // ties at the K-th value: do not compact every window
    tc.next_chk = t + window_span(n, tc.rate2, tc.span, span_max_at(t));
}

// Tile 0 of a row (kept out of line: it calls the threshold select).
template <int DT>
__device__ __forceinline__ void first_tile(const KParams& P, const int tid, const int r, RingPos& rp_io, Stream& st_io,
                                        const uint32_t U, TileCtx& tc_io) {
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    RingPos rp = rp_io;
    Stream st = st_io;
    TileCtx tc = tc_io;
    if (process_tile<DT, true>(P, p, g, tid, r, 0, rp, st, U, tc)) compact_window(P, tid, r, 0, st, tc, DT == FG_DTYPE_F32 ? 0 : DT);
    rp_io = rp;
    st_io = st;
    tc_io = tc;
}

// Tiles [t0, ntiles) of a row until a window end asks for a compaction.
// Contains no call, so the loop keeps its state in registers. Returns the
// next tile; *need tells whether a compaction is due first.
template <int DT>
__device__ __noinline__ int stream_row(const KParams& P, const int tid, const int r, const int t0, RingPos& rp_io,
                                       Stream& st_io, const uint32_t U, TileCtx& tc_io, bool& need) {
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<Elem<DT>::SIZE>(P, r);
    RingPos rp = rp_io;
    Stream st = st_io;
    TileCtx tc = tc_io;
    int t = t0;
    need = false;
    for (; t < g.ntiles; ++t) {
        if (process_tile<DT, false>(P, p, g, tid, r, t, rp, st, U, tc)) { need = true; ++t; break; }
    }
    rp_io = rp;
    st_io = st;
    tc_io = tc;
    return t;
}

__device__ __forceinline__ void release_claim(const KParams& P) {
    volatile uint32_t* go = &carve(smem_base(), P).ctl->go;
    *go = *go + 1u;
}

template <int DT>
__device__ void sample_row(const KParams& P, const int tid, const int r, RingPos& rp) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE, VEC = E::VEC;
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t ns = (uint32_t)P.nstage;
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<ESZ>(P, r);
    if (tid == 0) {
        RowCtl* ctl = carve(smem_base(), P).ctl;
        ctl->wcnt[0] = ctl->wcnt[1] = ctl->wcnt[2] = 0u;
        ctl->ovf[0] = ctl->ovf[1] = ctl->ovf[2] = 0;
        ctl->hikey = 0u; ctl->lokey = 0xffffffffu; ctl->xmin = -INFINITY;
        ctl->status = p.bad; ctl->nunique = 0u;
    }
    csync();
    if (p.pen) history_prologue_cold(P, tid, r);
    const uint32_t U = p.pen ? carve(smem_base(), P).ctl->nunique : 0u;
    Stream st;
    st.tmax = -INFINITY; st.imax = -INFINITY; st.itile = -1; st.tmin = INFINITY;
    st.zm = -1e30f; st.nzmc = -(st.zm * p.c); st.z0 = 0.0f; st.z1 = 0.0f;
    st.xmin = -INFINITY; st.cand = p.cand; st.base = 0; st.win = 0;
    st.bestv = -INFINITY; st.bestc = 0xffffffffu;
    st.khi = 0u; st.klo = 0xffffffffu;

    {
        const RowGeom gg = row_geom<ESZ>(P, r);
        TileCtx tc{-1, 0, 1, 0ull, (uint32_t)max(4 * p.K, 256)};
        if (gg.ntiles > 0) first_tile<DT>(P, tid, r, rp, st, U, tc);
        for (int t = 1; t < gg.ntiles;) {
            bool need;
            t = stream_row<DT>(P, tid, r, t, rp, st, U, tc, need);
            if (need) compact_window(P, tid, r, t - 1, st, tc, DT == FG_DTYPE_F32 ? 0 : DT);
        }
    }
    const bool heavy = row_heavy(P, r);

    const Smem s = carve(smem_base(), P);
    RowCtl* ctl = s.ctl;
    volatile int* abort = &ctl->abort;
    const uint8_t* rowp = reinterpret_cast<const uint8_t*>(P.logits) + (int64_t)r * P.row_stride * ESZ;
    // ---- ragged head/tail columns (at most 2 * (VEC - 1)), one per lane of warp 0;
    //      processed after the interior so the candidate filter is final ----
    if (warp == 0) {
        const int nh = g.head, nt = P.vocab - g.tail0;
        bool valid = lane < nh + nt;
        const int c = lane < nh ? lane : g.tail0 + (lane - nh);
        float x = -INFINITY;
        if (valid) {
            x = E::load(rowp, c);
            if (p.pen && (hist_bits(s, P.nwords, c, 1) & 1u)) {
                const uint32_t rk = hist_rank(s, (uint32_t)c);
                if (rk < U) s.sval[rk] = x;   // merged after the stream
                valid = false;
            }
        }
        process_one(p, s, st, x, (uint32_t)(valid ? c : 0), valid, lane);
    }

    // ---- merge the history columns with their penalised values ----
    if (p.pen) {
        csync();
        for (uint32_t i0 = 0; i0 < U; i0 += NCT) {
            const uint32_t i = i0 + tid;
            const bool valid = i < U;
            float x = -INFINITY;
            uint32_t col = 0;
            if (valid) { col = s.scol[i]; x = penalize(p, s, i, s.sval[i]); }
            process_one(p, s, st, x, col, valid, lane);
        }
    }
    // last window: nothing is appended after it, so only the limit applies
    if (st.cand) (void)window_check(P, r, p, s, tid, st, (uint32_t)HWM + (CAND_CAP - HWM) / 2, 1 << 20, 1);
    // uniform snapshot of the abort flag (the producer may set it at any time);
    // the ring position for the passes over the row that the finish may take
    if (tid == 0) { ctl->snap = (*abort != 0) ? 1u : 0u; ctl->rst = rp.st; ctl->rph = rp.ph; }
    csync();
    const bool aborted = ctl->snap != 0;

    finish_row_cold<DT>(P, tid, r, st.tmax, st.tmin, st.z0, st.z1, st.nzmc, st.cand, st.base, st.imax, st.itile,
                        st.bestv, st.bestc, aborted);
    csync();
    rp.st = ctl->rst;
    rp.ph = ctl->rph;
    // the row is done with: the producer may claim the next one
    if (tid == 0) release_claim(P);
    if (heavy) {
        // the producer streamed this row with an evict-last policy: release it
        const uintptr_t a0 = reinterpret_cast<uintptr_t>(g.interior) & ~uintptr_t(127);
        const uintptr_t a1 = reinterpret_cast<uintptr_t>(g.interior) + (uintptr_t)g.interior_bytes;
        for (uintptr_t a = a0 + (uintptr_t)tid * 128u; a < a1; a += (uintptr_t)NCT * 128u)
            l2_evict_normal(reinterpret_cast<const void*>(a));
    }
}

template <int DT>
__device__ void consumer(const KParams& P, const int tid) {
    RingPos rp{0u, 0u};
    uint32_t k = 0;
    while (true) {
        int r;
        {
            const Smem s = carve(smem_base(), P);
            RowCtl* ctl = s.ctl;
            volatile int* abort = &ctl->abort;
            const uint32_t slot = k % RQ, ph = (k / RQ) & 1u;
            if (tid == 0) {
                const bool ok = mbar_wait(&s.rowfull[slot], ph, abort);
                ctl->snap = ok ? (uint32_t)ctl->rowq[slot] : 0xfffffffeu;
            }
            csync();
            r = (int)ctl->snap;
            csync();
            if (tid == 0 && r != -2) mbar_arrive(&s.rowempty[slot]);
        }
        ++k;
        if (r < 0) break;
        sample_row<DT>(P, tid, r, rp);
        bool aborted;
        {
            const Smem s = carve(smem_base(), P);
            if (tid == 0) s.ctl->snap = (s.ctl->abort != 0) ? 1u : 0u;
            csync();
            aborted = s.ctl->snap != 0;
            csync();
        }
        if (aborted) break;
    }
    const Smem s = carve(smem_base(), P);
    RowCtl* ctl = s.ctl;
    volatile int* abort = &ctl->abort;
    if (tid == 0 && *abort) {
        // report the rows this CTA can no longer process: published ones, then the rest
        for (;; ++k) {
            const uint32_t slot = k % RQ, ph = (k / RQ) & 1u;
            if (!mbar_wait_for(&s.rowfull[slot], ph, 10000000ull)) break;
            const int rr = ctl->rowq[slot];
            mbar_arrive(&s.rowempty[slot]);
            if (rr < 0) break;
            P.out_ids[rr] = -1;
            if (P.out_status) P.out_status[rr] = FG_ROW_TIMEOUT;
        }
        for (;;) {
            const unsigned v = atomicAdd(&P.ws->next_row, 1u);
            if (v >= 2u * (unsigned)P.batch) break;
            if (!row_owned(P, v)) continue;   // handed out in the other half of the queue
            if (!row_wanted(P, (int)(v % (unsigned)P.batch))) continue;
            const unsigned rr = v % (unsigned)P.batch;
            P.out_ids[rr] = -1;
            if (P.out_status) P.out_status[rr] = FG_ROW_TIMEOUT;
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(NTHREADS, 2) fg_sample_kernel(const __grid_constant__ KParams P) {
    const Smem s = carve(smem_base(), P);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < P.nstage; ++i) { mbar_init(&s.full[i], 1); mbar_init(&s.empty[i], NCW); }
        for (int i = 0; i < RQ; ++i) { mbar_init(&s.rowfull[i], 1); mbar_init(&s.rowempty[i], 1); }
        s.ctl->abort = 0;
        s.ctl->go = 0u;
        s.ctl->preq = 0u;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid >= NCT) {
        if (tid == NCT) producer<DT>(P, s);
        return;
    }
    consumer<DT>(P, tid);
    // the last CTA to finish leaves the workspace zeroed for the next launch
    csync();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(&P.ws->done_ctas, 1u) == gridDim.x - 1) {
            P.ws->next_row = 0u;
            P.ws->done_ctas = 0u;
            __threadfence();
        }
    }
}

// ---------------------------------------------------------------------------
// Row argmax with torch.argmax semantics (first NaN, else first maximum).
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool arg_better(float a, uint32_t ia, float b, uint32_t ib) {
    const bool an = a != a, bn = b != b;
    if (an != bn) return an;
    if (!an && a != b) return a > b;
    return ia < ib;
}
template <int DT>
__global__ void __launch_bounds__(256) fg_argmax_kernel(const void* logits, int32_t V, int64_t stride, int64_t* out) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE, VEC = E::VEC;
    const int r = blockIdx.x, tid = threadIdx.x;
    const uint8_t* start = reinterpret_cast<const uint8_t*>(logits) + (int64_t)r * stride * ESZ;
    const uintptr_t a0 = (reinterpret_cast<uintptr_t>(start) + 15) & ~uintptr_t(15);
    const uintptr_t a1 = (reinterpret_cast<uintptr_t>(start) + (uintptr_t)V * ESZ) & ~uintptr_t(15);
    int head = V, tail0 = V;
    int64_t nchunk = 0;
    if (a1 > a0) {
        head = (int)((a0 - reinterpret_cast<uintptr_t>(start)) / ESZ);
        nchunk = (int64_t)(a1 - a0) / 16;
        tail0 = head + (int)(nchunk * VEC);
    }
    float bv = -INFINITY; uint32_t bi = 0xffffffffu;
    auto upd = [&](float v, uint32_t i) { if (bi == 0xffffffffu || arg_better(v, i, bv, bi)) { bv = v; bi = i; } };
    for (int c = tid; c < head; c += blockDim.x) upd(E::load(start, c), (uint32_t)c);
    for (int c = tail0 + tid; c < V; c += blockDim.x) upd(E::load(start, c), (uint32_t)c);
    const uint4* base = reinterpret_cast<const uint4*>(a0);
    for (int64_t ch = tid; ch < nchunk; ch += blockDim.x) {
        float x[VEC];
        E::unpack(__ldg(base + ch), x);
        const uint32_t c0 = (uint32_t)(head + ch * VEC);
#pragma unroll
        for (int e = 0; e < VEC; ++e) upd(x[e], c0 + e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi != 0xffffffffu && (bi == 0xffffffffu || arg_better(ov, oi, bv, bi))) { bv = ov; bi = oi; }
    }
    __shared__ float sv[8];
    __shared__ uint32_t si[8];
    if ((tid & 31) == 0) { sv[tid >> 5] = bv; si[tid >> 5] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (si[w] != 0xffffffffu && (bi == 0xffffffffu || arg_better(sv[w], si[w], bv, bi))) { bv = sv[w]; bi = si[w]; }
        out[r] = (int64_t)bi;
    }
}

// ---------------------------------------------------------------------------
// In-place repetition penalty (one CTA per row). The shared bitmap makes every
// unique id penalised exactly once, whatever its multiplicity in the history.
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) fg_rep_penalty_kernel(void* logits, int32_t V, int64_t stride,
                                                             const int32_t* hist_ids, const int64_t* hist_off,
                                                             const float* penalty) {
    using E = Elem<DT>;
    extern __shared__ uint32_t bm[];
    const int r = blockIdx.x, tid = threadIdx.x;
    const float pen = __ldg(penalty + r);
    if (pen == 1.0f) return;
    const int nw = (V + 31) / 32;
    for (int w = tid; w < nw; w += blockDim.x) bm[w] = 0u;
    __syncthreads();
    const int64_t h0 = __ldg(hist_off + r), h1 = __ldg(hist_off + r + 1);
    uint8_t* row = reinterpret_cast<uint8_t*>(logits) + (int64_t)r * stride * E::SIZE;
    for (int64_t i = h0 + tid; i < h1; i += blockDim.x) {
        const int32_t c = __ldg(hist_ids + i);
        if (c < 0 || c >= V) continue;
        const uint32_t bit = 1u << (c & 31);
        const uint32_t old = atomicOr(&bm[c >> 5], bit);
        if (!(old & bit)) {
            const float x = E::load(row, c);
            const float y = (x > 0.0f) ? __fdiv_rn(x, pen) : __fmul_rn(x, pen);
            E::store(row, c, y);
        }
    }
}

}  // namespace fg
