// fg_kernels.cuh — kernels behind the C ABI in include/flashgen_sampler.h.
//
//   fg_sample_kernel<DT>      fused penalties/temperature/top-k/top-p/draw
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

__device__ __forceinline__ uint32_t& word_of(uint4& v, int q) {
    return q == 0 ? v.x : (q == 1 ? v.y : (q == 2 ? v.z : v.w));
}
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
template <int DT>
__device__ __forceinline__ void elem_mask(uint4& v, int e) {
    if constexpr (DT == FG_DTYPE_F32) {
        word_of(v, e) = Neg<DT>::W;
    } else {
        uint32_t& w = word_of(v, e >> 1);
        w = (e & 1) ? ((w & 0x0000ffffu) | (Neg<DT>::W & 0xffff0000u)) : ((w & 0xffff0000u) | (Neg<DT>::W & 0xffffu));
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
    const int64_t h0 = __ldg(P.hist_offsets + r), h1 = __ldg(P.hist_offsets + r + 1);
    constexpr int HB = 4;   // ids per thread per batch, loaded together
    int bad = 0;
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
            if (i >= h1) continue;
            const int64_t gid = ids[j];
            if (gid < 0 || gid >= P.vocab_total) { bad = 1; continue; }
            const int64_t c = gid - P.vocab_offset;
            if (c >= 0 && c < P.vocab) {
                const uint32_t bit = 1u << (c & 31);
                if (!(s.bitmap[c >> 5] & bit)) atomicOr(&s.bitmap[c >> 5], bit);
            }
        }
    }
    if (bad) atomicOr(&s.ctl->status, FG_ROW_BAD_HISTORY);
    csync();
    // thread t owns the word pairs [q0, q1): prefix counts and the scol entries
    const int ppt = (npair + NCT - 1) / NCT;
    const int q0 = tid * ppt, q1 = min(npair, q0 + ppt);
    uint32_t local = 0;
    for (int q = q0; q < q1; ++q) {
        local += __popc(s.bitmap[2 * q]);
        if (2 * q + 1 < nw) local += __popc(s.bitmap[2 * q + 1]);
    }
    uint32_t total;
    uint32_t run = cons_excl_scan_u32(local, total, s, tid);
    const uint32_t cap = (uint32_t)P.hu_cap;
    for (int q = q0; q < q1; ++q) {
        s.prefix[q] = (uint16_t)run;
        run += __popc(s.bitmap[2 * q]) + (2 * q + 1 < nw ? __popc(s.bitmap[2 * q + 1]) : 0);
    }
    csync();
    // ascending list of distinct columns: words strided over the threads
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
    const uint32_t U = min(total, cap);
    if (tid == 0) {
        s.ctl->nunique = U;
        if (total > cap || total > 65535u) atomicOr(&s.ctl->status, FG_ROW_BAD_PARAM);
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
                const int64_t c = gid - P.vocab_offset;
                bool v = i < h1 && gid >= 0 && gid < P.vocab_total && c >= 0 && c < P.vocab;
                const uint32_t rk = v ? hist_rank(s, (uint32_t)c) : 0u;
                v = v && rk < U;
                if (v) atomicAdd(&s.counts[rk], 1u);
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
    const uint32_t pos = st.base + atomicAdd(&s.ctl->wcnt[slot], 1u);
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
__device__ uint32_t compact(const RowParams& p, const Smem& s, int tid, uint32_t n, Stream& st) {
    RowCtl* ctl = s.ctl;
    if (n <= (uint32_t)p.K) return n;
    const uint32_t lo = cons_min_u32(st.klo, s, tid), hi = cons_max_u32(st.khi, s, tid);
    if (lo > hi) return n;
    const SelOut so = block_select<true, true>(
        [&](auto&& f) {
            for (uint32_t i0 = 0; i0 < n; i0 += NCT) {
                const uint32_t i = i0 + tid;
                f(i < n, i < n ? s.ckey[i] : 0u, 1ull);
            }
        },
        (uint64_t)(p.K - 1), lo, varying_bits(lo, hi), s, tid);
    if (!so.ok) return n;
    if (tid == 0) {
        const float xm = xmin_for(p, funkey(so.key));
        if (xm > ctl->xmin) ctl->xmin = xm;
    }
    csync();
    const uint32_t kmin = fkey(ctl->xmin);
    st.klo = max(st.klo, kmin);
    uint32_t out = 0;
    for (uint32_t base = 0; base < n; base += NCT * 8) {
        uint32_t kk[8], ii[8], keep = 0, cnt = 0;
        const uint32_t i0 = base + tid * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t idx = i0 + j;
            kk[j] = idx < n ? s.ckey[idx] : 0u;
            ii[j] = idx < n ? s.cid[idx] : 0u;
            if (idx < n && kk[j] >= kmin) { keep |= 1u << j; ++cnt; }
        }
        uint32_t total;
        uint32_t pos = out + cons_excl_scan_u32(cnt, total, s, tid);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (keep >> j & 1u) { s.ckey[pos] = kk[j]; s.cid[pos] = ii[j]; ++pos; }
        out += total;
        csync();
    }
    return out;
}

// End of a candidate window: uniform candidate count, compaction when the
// buffer passed `limit`.
__device__ __forceinline__ void window_check(const RowParams& p, const Smem& s, int tid, Stream& st, uint32_t limit) {
    csync();
    const int slot = (int)(st.win % 3u);
    uint32_t n = st.base + s.ctl->wcnt[slot];
    const bool ovf = s.ctl->ovf[slot] != 0;
    if (tid == 0) { s.ctl->wcnt[(slot + 2) % 3] = 0u; s.ctl->ovf[(slot + 2) % 3] = 0; }
    st.win += 1;
    if (st.cand) {
        if (ovf) {
            st.cand = false;
        } else if (n > limit) {
            n = compact(p, s, tid, n, st);
            if (n > limit) st.cand = false;
        }
        st.xmin = s.ctl->xmin;
    }
    st.base = n;
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
    const int64_t nchunk = g.interior_bytes / 16;
    for (int64_t ch0 = 0; ch0 < nchunk; ch0 += NCT) {
        const int64_t ch = ch0 + tid;
        const bool valid = ch < nchunk;
        float x[VEC];
        int c0 = 0;
        if (valid) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(g.interior) + ch);
            E::unpack(v, x);
            c0 = g.head + (int)(ch * VEC);
            if (p.pen) {
                uint32_t bits = hist_bits(s, P.nwords, c0, VEC);
                while (bits) {
                    const int e = __ffs(bits) - 1;
                    bits &= bits - 1;
                    const uint32_t rk = hist_rank(s, (uint32_t)(c0 + e));
#pragma unroll
                    for (int j = 0; j < VEC; ++j)
                        if (j == e) x[j] = penalize(p, s, rk, x[j]);
                }
            }
        } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) x[e] = -INFINITY;
        }
#pragma unroll
        for (int e = 0; e < VEC; ++e) f(valid, c0 + e, x[e]);
    }
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
__device__ Located locate(const KParams& P, const Smem& s, const RowParams& p, int r, const RowGeom& g, int tid,
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
            const uint32_t pos = slot0 + atomicAdd(&s.ctl->ncol, 1u);
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
    volatile int* abort = &s.ctl->abort;
    const uint32_t ns = (uint32_t)P.nstage;
    uint32_t it = 0, k = 0, st = 0, ph = 0;
    auto fetch = [&]() -> int {
        const unsigned v = atomicAdd(&P.ws->next_row, 1u);
        return v < (unsigned)P.batch ? (int)v : -1;
    };
    auto drain = [&]() {
        const uint32_t first = it > ns ? it - ns : 0u;
        for (uint32_t j = first; j < it; ++j) mbar_wait_for(&s.full[j % ns], (j / ns) & 1u, WAIT_LIMIT_NS);
    };
    auto give_up = [&](int rr) {
        *abort = 1;
        if (rr >= 0) { P.out_ids[rr] = -1; if (P.out_status) P.out_status[rr] = FG_ROW_TIMEOUT; }
        drain();
    };
    int r = fetch();
    while (true) {
        const uint32_t slot = k % RQ, rph = (k / RQ) & 1u;
        if (!mbar_wait(&s.rowempty[slot], rph ^ 1u, abort)) { give_up(r); return; }
        s.ctl->rowq[slot] = r;
        mbar_arrive(&s.rowfull[slot]);
        ++k;
        if (r < 0) return;
        const int rcur = r;
        r = fetch();  // next row index, fetched while this row streams
        const RowGeom g = row_geom<ESZ>(P, rcur);
        for (int t = 0; t < g.ntiles; ++t, ++it) {
            if (!mbar_wait(&s.empty[st], ph ^ 1u, abort)) { give_up(r); return; }
            const int64_t off = (int64_t)t * TILE_BYTES;
            const int64_t left = g.interior_bytes - off;
            const uint32_t bytes = (uint32_t)(left < TILE_BYTES ? left : TILE_BYTES);
            mbar_arrive_expect_tx(&s.full[st], bytes);
            bulk_g2s(s.ring + (int64_t)st * TILE_BYTES, g.interior + off, bytes, &s.full[st]);
            if (++st == ns) { st = 0; ph ^= 1u; }
        }
    }
}

// ---------------------------------------------------------------------------
// Consumer warps: one row
// ---------------------------------------------------------------------------
struct RingPos { uint32_t st, ph; };

template <int DT>
__device__ void sample_row(const KParams& P, const Smem& s, const int tid, const int r, RingPos& rp) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE, VEC = E::VEC;
    const int lane = tid & 31, warp = tid >> 5;
    RowCtl* ctl = s.ctl;
    volatile int* abort = &ctl->abort;
    const uint32_t ns = (uint32_t)P.nstage;
    const float scale = __uint_as_float((uint32_t)(127 + P.mass_shift) << 23);  // 2^S
    const RowParams p = row_params(P, r);
    const RowGeom g = row_geom<ESZ>(P, r);
    if (tid == 0) {
        ctl->wcnt[0] = ctl->wcnt[1] = ctl->wcnt[2] = 0u;
        ctl->ovf[0] = ctl->ovf[1] = ctl->ovf[2] = 0;
        ctl->hikey = 0u; ctl->lokey = 0xffffffffu; ctl->xmin = -INFINITY;
        ctl->status = p.bad; ctl->nunique = 0u;
    }
    csync();
    if (p.pen) history_prologue(P, s, p, r, tid);
    const uint32_t U = p.pen ? ctl->nunique : 0u;
    Stream st;
    st.tmax = -INFINITY; st.imax = -INFINITY; st.itile = -1; st.tmin = INFINITY;
    st.zm = -1e30f; st.nzmc = -(st.zm * p.c); st.z0 = 0.0f; st.z1 = 0.0f;
    st.xmin = -INFINITY; st.cand = p.cand; st.base = 0; st.win = 0;
    st.bestv = -INFINITY; st.bestc = 0xffffffffu;
    st.khi = 0u; st.klo = 0xffffffffu;
    const uint8_t* rowp = reinterpret_cast<const uint8_t*>(P.logits) + (int64_t)r * P.row_stride * ESZ;

    // ---- streamed interior ----
    for (int t = 0; t < g.ntiles; ++t) {
        const bool ok = mbar_wait(&s.full[rp.st], rp.ph, abort);
        if (!ok) *abort = 1;
        const uint8_t* tile = s.ring + (int64_t)rp.st * TILE_BYTES;
        const int64_t left = g.interior_bytes - (int64_t)t * TILE_BYTES;
        const int nch = ok ? (int)((left < TILE_BYTES ? left : TILE_BYTES) / 16) : 0;
        const int tcol0 = g.head + t * (TILE_BYTES / ESZ);
        uint4 v[CPT];
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            const int ch = tid + j * NCT;
            if (ch < nch) v[j] = *reinterpret_cast<const uint4*>(tile + ch * 16);
            else v[j] = make_uint4(Neg<DT>::W, Neg<DT>::W, Neg<DT>::W, Neg<DT>::W);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[rp.st]);   // the stage now lives in registers
        if (++rp.st == ns) { rp.st = 0; rp.ph ^= 1u; }
        uint32_t hb[CPT];
#pragma unroll
        for (int j = 0; j < CPT; ++j) hb[j] = 0u;
        if (p.pen) {
#pragma unroll
            for (int j = 0; j < CPT; ++j) {
                const int ch = tid + j * NCT;
                if (ch < nch) {
                    const int c0 = tcol0 + ch * VEC;
                    uint32_t bits = hist_bits(s, P.nwords, c0, VEC);
                    hb[j] = bits;
                    while (bits) {
                        const int e = __ffs(bits) - 1;
                        bits &= bits - 1;
                        const uint32_t rk = hist_rank(s, (uint32_t)(c0 + e));
                        if (rk < U) s.sval[rk] = elem_get<DT>(v[j], e);
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
            if (t == 0) {
                // starting threshold from the first tile: the K-th largest of
                // disjoint group maxima (thread maxima for K <= NCT/2, chunk
                // maxima for K <= NCT, elements otherwise) bounds the row's K-th
                // largest from below
                float cm[CPT];
#pragma unroll
                for (int j = 0; j < CPT; ++j) cm[j] = chunk_max1<DT>(v[j]);
                const int K = p.K;
                // key range of the values the select will see
                float lo_v = INFINITY;
                if (K <= NCT / 2) lo_v = m;
                else if (K <= NCT) { for (int j = 0; j < CPT; ++j) lo_v = fminf(lo_v, cm[j]); }
                else lo_v = chunks_min<DT>(v);
                const uint32_t klo = cons_min_u32((lo_v == lo_v && lo_v > -INFINITY) ? fkey(lo_v) : 0xffffffffu, s, tid);
                const uint32_t khi = cons_max_u32((m == m && m > -INFINITY) ? fkey(m) : 0u, s, tid);
                const SelOut so = block_select<true, true>(
                    [&](auto&& f) {
                        if (K <= NCT / 2) {
                            f(m == m && m > -INFINITY, fkey(m), 1ull);
                        } else if (K <= NCT) {
#pragma unroll
                            for (int j = 0; j < CPT; ++j) f(cm[j] == cm[j] && cm[j] > -INFINITY, fkey(cm[j]), 1ull);
                        } else {
#pragma unroll
                            for (int j = 0; j < CPT; ++j)
#pragma unroll
                                for (int e = 0; e < VEC; ++e) {
                                    const float x = elem_get<DT>(v[j], e);
                                    f(x == x && x > -INFINITY, fkey(x), 1ull);
                                }
                        }
                    },
                    (uint64_t)(K - 1), klo <= khi ? klo : 0u, klo <= khi ? varying_bits(klo, khi) : 32, s, tid);
                if (so.ok && tid == 0) {
                    const float xm = xmin_for(p, funkey(so.key));
                    if (xm > ctl->xmin) ctl->xmin = xm;
                }
                csync();
                st.xmin = ctl->xmin;
            }
            uint32_t pick = 0;
            if (m >= st.xmin) {
#pragma unroll
                for (int j = 0; j < CPT; ++j) {
                    const int ch = tid + j * NCT;
                    if (ch < nch) {
#pragma unroll
                        for (int e = 0; e < VEC; ++e)
                            if (!((hb[j] >> e) & 1u) && elem_get<DT>(v[j], e) >= st.xmin) pick |= 1u << (j * VEC + e);
                    }
                }
            }
            while (pick) {
                const int i = __ffs(pick) - 1;
                pick &= pick - 1;
                const int j = i / VEC, e = i % VEC;
                uint4 vv = v[0];
#pragma unroll
                for (int jj = 1; jj < CPT; ++jj) if (jj == j) vv = v[jj];
                append1(s, st, fkey(elem_get<DT>(vv, e)), (uint32_t)(tcol0 + (tid + j * NCT) * VEC + e));
            }
            // appends per tile fall off as 1/t: check every tile early in the
            // row, every 2nd and then every 4th tile later (appends are bounds
            // checked, an overflow sends the row to the multi-pass path)
            const bool chk = t < 8 || (t < 16 ? (t & 1) == 1 : (t & 3) == 3) || t == g.ntiles - 1;
            if (chk) window_check(p, s, tid, st, (uint32_t)HWM);
        }
    }

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
    if (st.cand) window_check(p, s, tid, st, (uint32_t)HWM + (CAND_CAP - HWM) / 2);
    // uniform snapshot of the abort flag (the producer may set it at any time)
    if (tid == 0) ctl->snap = (*abort != 0) ? 1u : 0u;
    csync();
    const bool aborted = ctl->snap != 0;

    // ---- row statistics ----
    const float M = cons_max_nan(st.tmax, s, tid);
    int status = ctl->status;
    const bool cand_ok = st.cand && !aborted;
    const uint32_t n = st.base;
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
    int64_t out_id = -1;
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
        // top-k threshold (on C, or over the whole row when C cannot hold it)
        uint32_t ykK = 0u;
        if (p.mode == MODE_TOPK) {
            if (cand_ok) {
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
        uint64_t loc = 0;
        for (uint32_t i = tid; i < nC; i += NCT) if (keepk(s.ckey[i])) loc += qC(s.ckey[i]);
        const uint64_t AC = cons_sum_u64(loc, s, tid);   // exact mass of the kept part of C

        // region R below C (whole row when C is empty), restricted to y >= T_K for top-k
        const uint32_t rlo = (p.mode == MODE_TOPK) ? ykK : KEY_NEG_INF;
        const uint32_t rhi = nC > 0 ? loY - 1u : 0xffffffffu;
        const float yRlo = (p.mode == MODE_TOPK) ? fmaxf(funkey(ykK), My - 64.0f) : ymin;
        const float yRhi = nC > 0 ? funkey(loY - 1u) : My;
        bool cut = false, cut_in_R = false;
        uint32_t tstar = 0u, id_cut = 0xffffffffu;
        uint64_t Qf = 0, m_t = 0, n_t = 0;
        if (p.use_p) {
            double Qn;
            if (p.mode == MODE_TOPK && cand_ok) Qn = (double)AC;
            else if (p.mode == MODE_TOPK) {
                const Located L0 = locate<DT>(P, s, p, r, g, tid, rlo, rhi, yRlo, yRhi, 0ull, My, scale, 0u);
                Qn = (double)L0.total;
            } else Qn = Zq;
            const double Pd = (double)p.top_p * Qn;
            const uint64_t Pt = (uint64_t)floor(Pd);
            cut = true;
            if ((double)AC > Pd && nC > 0) {
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
                const Located L = locate<DT>(P, s, p, r, g, tid, rlo, rhi, yRlo, yRhi, tr, My, scale, nC);
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
                const Located L0 = locate<DT>(P, s, p, r, g, tid, rlo, rhi, yRlo, yRhi, 0ull, My, scale, 0u);
                Qf = L0.total;
            } else Qf = (uint64_t)Zq;   // unfiltered: every token kept
        }
        // ---- inverse-CDF draw in descending-probability order ----
        if (Qf > 0) {
            uint64_t target = (uint64_t)floor((double)p.u * (double)Qf);
            if (target >= Qf) target = Qf - 1;
            if (target < AC && nC > 0) {
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
                }
            } else {
                status |= FG_ROW_GENERAL_PATH;
                const uint64_t t2 = target - (nC > 0 ? AC : 0ull);
                const uint32_t rlo2 = cut_in_R ? tstar : rlo;
                const float ylo2 = cut_in_R ? fmaxf(funkey(tstar), My - 64.0f) : yRlo;
                const Located L = locate<DT>(P, s, p, r, g, tid, rlo2, rhi, ylo2, yRhi, t2, My, scale, nC);
                if (L.ok) {
                    const uint64_t qd = L.n_at ? L.at / L.n_at : 0;
                    uint64_t j = qd ? (t2 - L.before) / qd : 0;
                    if (j >= L.n_at) j = L.n_at ? L.n_at - 1 : 0;
                    out_id = L.in_buffer ? jth_id(P, s, tid, L.n0, L.n1, L.key, L.n_at, j)
                                         : jth_id_row<DT>(P, s, p, r, g, tid, L.key, j);
                }
            }
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
    }
    if (pr && out_id < 0) for (int c = tid; c < P.vocab; c += NCT) pr[c] = 0.0f;
    if (tid == 0) {
        P.out_ids[r] = (out_id >= 0) ? out_id + P.vocab_offset : -1;
        if (P.out_status) P.out_status[r] = status;
    }
    csync();
    if (aborted && tid == 0) *abort = 1;
}

template <int DT>
__device__ void consumer(const KParams& P, const Smem& s, const int tid) {
    RowCtl* ctl = s.ctl;
    volatile int* abort = &ctl->abort;
    RingPos rp{0u, 0u};
    uint32_t k = 0;
    while (true) {
        const uint32_t slot = k % RQ, ph = (k / RQ) & 1u;
        if (tid == 0) {
            const bool ok = mbar_wait(&s.rowfull[slot], ph, abort);
            ctl->snap = ok ? (uint32_t)ctl->rowq[slot] : 0xfffffffeu;
        }
        csync();
        const int r = (int)ctl->snap;
        csync();
        if (tid == 0 && r != -2) mbar_arrive(&s.rowempty[slot]);
        ++k;
        if (r < 0) break;
        sample_row<DT>(P, s, tid, r, rp);
        if (tid == 0) ctl->snap = (*abort != 0) ? 1u : 0u;
        csync();
        const bool aborted = ctl->snap != 0;
        csync();
        if (aborted) break;
    }
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
            if (v >= (unsigned)P.batch) break;
            P.out_ids[v] = -1;
            if (P.out_status) P.out_status[v] = FG_ROW_TIMEOUT;
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(NTHREADS, 2) fg_sample_kernel(const KParams P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem s = carve(smem_raw, P);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < P.nstage; ++i) { mbar_init(&s.full[i], 1); mbar_init(&s.empty[i], NCW); }
        for (int i = 0; i < RQ; ++i) { mbar_init(&s.rowfull[i], 1); mbar_init(&s.rowempty[i], 1); }
        s.ctl->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid >= NCT) {
        if (tid == NCT) producer<DT>(P, s);
        return;
    }
    consumer<DT>(P, s, tid);
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
