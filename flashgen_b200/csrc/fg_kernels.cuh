// fg_kernels.cuh — kernels behind the C ABI in include/flashgen_sampler.h.
//
//   fg_sample_kernel<DT>      fused penalties/temperature/top-k/top-p/draw
//   fg_argmax_kernel<DT>      row argmax (torch.argmax semantics)
//   fg_rep_penalty_kernel<DT> in-place repetition penalty
#pragma once
#include "fg_sample_kernel.cuh"

namespace fg {

// ---------------------------------------------------------------------------
// History prologue: bitmap of this row's history ids restricted to the
// columns of this call; when a frequency penalty is set, also the rank of
// every set bit (word prefix of popcounts) and the count of each id.
// ---------------------------------------------------------------------------
__device__ void history_prologue(const KParams& P, const Smem& s, const RowParams& p, int r, int tid) {
    const int nw = P.nwords;
    for (int w = tid; w < nw; w += NCT) s.bitmap[w] = 0u;
    csync();
    const int64_t h0 = __ldg(P.hist_offsets + r), h1 = __ldg(P.hist_offsets + r + 1);
    int bad = 0;
    for (int64_t i = h0 + tid; i < h1; i += NCT) {
        const int64_t gid = __ldg(P.hist_ids + i);
        if (gid < 0 || gid >= P.vocab_total) { bad = 1; continue; }
        const int64_t c = gid - P.vocab_offset;
        if (c >= 0 && c < P.vocab) atomicOr(&s.bitmap[c >> 5], 1u << (c & 31));
    }
    if (bad) atomicOr(&s.ctl->status, FG_ROW_BAD_HISTORY);
    csync();
    if (!p.freq_on) return;
    // word prefix of popcounts: thread t owns a contiguous range of words
    const int wpt = (nw + NCT - 1) / NCT;
    const int w0 = tid * wpt, w1 = min(nw, w0 + wpt);
    uint32_t local = 0;
    for (int w = w0; w < w1; ++w) local += __popc(s.bitmap[w]);
    uint32_t total;
    uint32_t run = cons_excl_scan_u32(local, total, s, tid);
    for (int w = w0; w < w1; ++w) { s.prefix[w] = run; run += __popc(s.bitmap[w]); }
    const uint32_t U = min(total, (uint32_t)P.hu_cap);
    for (uint32_t i = tid; i < U; i += NCT) s.counts[i] = 0u;
    if (tid == 0 && total > (uint32_t)P.hu_cap) atomicOr(&s.ctl->status, FG_ROW_BAD_PARAM);
    csync();
    for (int64_t i = h0 + tid; i < h1; i += NCT) {
        const int64_t gid = __ldg(P.hist_ids + i);
        if (gid < 0 || gid >= P.vocab_total) continue;
        const int64_t c = gid - P.vocab_offset;
        if (c < 0 || c >= P.vocab) continue;
        const uint32_t w = (uint32_t)(c >> 5), b = (uint32_t)(c & 31);
        const uint32_t rank = s.prefix[w] + __popc(s.bitmap[w] & ((1u << b) - 1u));
        if (rank < (uint32_t)P.hu_cap) atomicAdd(&s.counts[rank], 1u);
    }
    csync();
}

// Penalised value of column c (its history bit is known to be set).
__device__ __forceinline__ float penalize(const RowParams& p, const Smem& s, int c, float x) {
    if (p.rep_on) x = (x > 0.0f) ? __fdiv_rn(x, p.rep) : __fmul_rn(x, p.rep);
    if (p.freq_on) {
        const uint32_t w = (uint32_t)c >> 5, b = (uint32_t)c & 31;
        const uint32_t rank = s.prefix[w] + __popc(s.bitmap[w] & ((1u << b) - 1u));
        const float cnt = (float)s.counts[rank];
        x = __fsub_rn(x, __fmul_rn(p.freq, cnt));
    }
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
template <int N>
__device__ __forceinline__ void penalize_chunk(const RowParams& p, const Smem& s, int nwords, int c0, float (&x)[N]) {
    uint32_t bits = hist_bits(s, nwords, c0, N);
    while (bits) {
        const int e = __ffs(bits) - 1;
        bits &= bits - 1;
#pragma unroll
        for (int j = 0; j < N; ++j) if (j == e) x[j] = penalize(p, s, c0 + j, x[j]);
    }
}

__device__ __forceinline__ float ex2_approx(float v) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(v));
    return y;
}

// ---------------------------------------------------------------------------
// Streaming state of one consumer thread
// ---------------------------------------------------------------------------
struct Stream {
    float tmax;    // NaN-propagating max of penalised x
    float zm;      // running max used by the online sum-exp
    float zmc;     // fl(zm * c)
    float z;       // sum of 2^(x*c - zmc)
    float xmin;    // register copy of the candidate filter
    bool cand;
};

// Process N values x[0..N) of columns cols(e) = c0 + e (valid bits in vmask).
template <int N>
__device__ __forceinline__ void process(const RowParams& p, const Smem& s, Stream& st, const float (&x)[N],
                                        int c0, uint32_t vmask, int lane) {
    float cmax = -INFINITY;
#pragma unroll
    for (int e = 0; e < N; ++e) if (vmask >> e & 1u) cmax = fmax_nan(cmax, x[e]);
    st.tmax = fmax_nan(st.tmax, cmax);
    if (p.mode == MODE_NUCLEUS) {
        if (cmax > st.zm) {
            const float nmc = cmax * p.c;
            st.z *= ex2_approx(st.zmc - nmc);
            st.zm = cmax; st.zmc = nmc;
        }
#pragma unroll
        for (int e = 0; e < N; ++e)
            if (vmask >> e & 1u) st.z += ex2_approx(__fmaf_rn(x[e], p.c, -st.zmc));
    }
    if (st.cand) {
        uint32_t pm = 0;
#pragma unroll
        for (int e = 0; e < N; ++e) if ((vmask >> e & 1u) && x[e] >= st.xmin) pm |= 1u << e;
        if (__any_sync(0xffffffffu, pm)) {
            const uint32_t cnt = __popc(pm);
            const uint32_t incl = warp_incl_scan_u32(cnt, lane);
            const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
            uint32_t base = 0;
            if (lane == 31) base = atomicAdd(&s.ctl->n, total);
            base = __shfl_sync(0xffffffffu, base, 31);
            uint32_t pos = base + incl - cnt;
            uint32_t kmax = 0;
#pragma unroll
            for (int e = 0; e < N; ++e) {
                if (pm >> e & 1u) {
                    const uint32_t k = fkey(x[e]);
                    if (pos < (uint32_t)CAND_CAP) { s.ckey[pos] = k; s.cid[pos] = (uint32_t)(c0 + e); }
                    ++pos;
                    kmax = max(kmax, k);
                }
            }
            kmax = __reduce_max_sync(0xffffffffu, kmax);
            if (lane == 0) atomicMax(&s.ctl->hikey, kmax);
        }
    }
}

// ---------------------------------------------------------------------------
// Compaction: raise xmin to a valid lower bound of the K-th largest value and
// drop candidates below it (stable, in place).
// ---------------------------------------------------------------------------
__device__ void compact(const RowParams& p, const Smem& s, int tid, uint32_t n) {
    RowCtl* ctl = s.ctl;
    const uint32_t lo = fkey(ctl->xmin);
    const uint32_t hi = ctl->hikey;
    const uint32_t span = hi >= lo ? hi - lo : 0u;
    const int shift = span < (uint32_t)NBINS ? 0 : (32 - __clz(span) - 8);
    if (tid < NBINS) s.cnts[tid] = 0u;
    csync();
    for (uint32_t i = tid; i < n; i += NCT) {
        const uint32_t k = s.ckey[i];
        if (k >= lo) atomicAdd(&s.cnts[(k - lo) >> shift], 1u);
    }
    csync();
    if (tid < 32) {
        const int lane = tid;
        uint32_t v[8], lsum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) { v[j] = s.cnts[NBINS - 1 - (lane * 8 + j)]; lsum += v[j]; }
        const uint32_t incl = warp_incl_scan_u32(lsum, lane);
        const uint32_t excl = incl - lsum;
        const uint32_t K = (uint32_t)p.K;
        const bool mine = excl < K && K <= incl;
        const uint32_t bal = __ballot_sync(0xffffffffu, mine);
        if (bal != 0 && lane == __ffs(bal) - 1) {
            uint32_t c = excl;
            int jj = 0;
            for (; jj < 7; ++jj) { c += v[jj]; if (c >= K) break; }
            const uint32_t b = (uint32_t)(NBINS - 1 - (lane * 8 + jj));
            const uint32_t tau_key = lo + (b << shift);
            const float xm = xmin_for(p, funkey(tau_key));
            if (xm > ctl->xmin) ctl->xmin = xm;
        }
    }
    csync();
    const uint32_t kmin = fkey(ctl->xmin);
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
    if (tid == 0) {
        ctl->n = out;
        if (out > (uint32_t)HWM) { ctl->cand_on = 0; ctl->general = 1; }
    }
    csync();
}

// ---------------------------------------------------------------------------
// Whole-row enumeration from global memory (general path).
// f(col, x) with x the penalised fp32 value.
// ---------------------------------------------------------------------------
template <int DT, class F>
__device__ __forceinline__ void for_row(const KParams& P, const Smem& s, const RowParams& p, int r,
                                        const RowGeom& g, int tid, F&& f) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE, VEC = E::VEC;
    const uint8_t* row = reinterpret_cast<const uint8_t*>(P.logits) + (int64_t)r * P.row_stride * ESZ;
    const int nh = g.head, nt = P.vocab - g.tail0;
    if (tid < nh + nt) {
        const int c = tid < nh ? tid : g.tail0 + (tid - nh);
        float x = E::load(row, c);
        if (p.pen && (hist_bits(s, P.nwords, c, 1) & 1u)) x = penalize(p, s, c, x);
        f(c, x);
    }
    const int64_t nchunk = g.interior_bytes / 16;
    for (int64_t ch = tid; ch < nchunk; ch += NCT) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(g.interior) + ch);
        float x[VEC];
        E::unpack(v, x);
        const int c0 = g.head + (int)(ch * (16 / ESZ));
        if (p.pen) penalize_chunk<VEC>(p, s, P.nwords, c0, x);
#pragma unroll
        for (int e = 0; e < VEC; ++e) f(c0 + e, x[e]);
    }
}

__device__ __forceinline__ uint64_t mass_q(float y, float My, float scale) {
    const float e = expf(y - My);
    return (uint64_t)__float2ull_rn(e * scale);
}

// ---------------------------------------------------------------------------
// Sampling decision over an abstract element set.
//   enumerate(f): f(ykey, col, q, keep_k) for the thread's elements
// Returns the chosen column (or -1 if the set is empty), fills probs.
// ---------------------------------------------------------------------------
template <class Enum>
__device__ int decide(const KParams& P, const Smem& s, const RowParams& p, int r, int tid,
                      Enum&& enumerate, bool topk_done, uint32_t ykK, double Qn_override, bool* not_covered) {
    *not_covered = false;
    // kept_k predicate: y >= ykK (TOPK) or every element
    auto keep_k = [&](uint32_t yk) { return !topk_done || yk >= ykK; };
    uint64_t myq = 0;
    enumerate([&](uint32_t yk, uint32_t col, uint64_t q) { if (keep_k(yk)) myq += q; });
    const uint64_t Qk = cons_sum_u64(myq, s, tid);
    uint32_t tstar = 0, id_cut = 0xffffffffu;
    bool pcut = false, partial = false;
    if (p.use_p) {
        const double Qn = Qn_override > 0.0 ? Qn_override : (double)Qk;
        const double Pd = (double)p.top_p * Qn;
        if ((double)Qk <= Pd) { *not_covered = true; return -1; }
        const uint64_t Pt = (uint64_t)floor(Pd);
        SelOut so = block_select<true, false>(
            [&](auto&& f) { enumerate([&](uint32_t yk, uint32_t col, uint64_t q) { if (keep_k(yk)) f(yk, q); }); },
            Pt, 32, s, tid);
        if (!so.ok) { *not_covered = true; return -1; }
        tstar = so.key;
        pcut = true;
        const uint64_t qt = so.n_at ? so.at / so.n_at : 0;
        uint64_t m = so.n_at;
        if (qt > 0) { const uint64_t mm = (Pt - so.before) / qt + 1; if (mm < m) m = mm; }
        if (m < so.n_at) {
            partial = true;
            SelOut si = block_select<false, true>(
                [&](auto&& f) { enumerate([&](uint32_t yk, uint32_t col, uint64_t q) { if (yk == tstar) f(col, 1); }); },
                m - 1, P.id_bits, s, tid);
            id_cut = si.key;
        }
    }
    auto keep_f = [&](uint32_t yk, uint32_t col) {
        if (!keep_k(yk)) return false;
        if (!pcut) return true;
        if (yk > tstar) return true;
        if (yk < tstar) return false;
        return !partial || col <= id_cut;
    };
    myq = 0;
    enumerate([&](uint32_t yk, uint32_t col, uint64_t q) { if (keep_f(yk, col)) myq += q; });
    const uint64_t Qf = cons_sum_u64(myq, s, tid);
    if (Qf == 0) return -1;
    uint64_t target = (uint64_t)floor((double)p.u * (double)Qf);
    if (target >= Qf) target = Qf - 1;
    SelOut sd = block_select<false, false>(
        [&](auto&& f) { enumerate([&](uint32_t yk, uint32_t col, uint64_t q) { if (keep_f(yk, col)) f(col, q); }); },
        target, P.id_bits, s, tid);
    if (P.out_probs) {
        float* pr = P.out_probs + (int64_t)r * P.vocab;
        for (int c = tid; c < P.vocab; c += NCT) pr[c] = 0.0f;
        csync();
        const double inv = 1.0 / (double)Qf;
        enumerate([&](uint32_t yk, uint32_t col, uint64_t q) {
            if (keep_f(yk, col)) pr[col] = (float)((double)q * inv);
        });
        csync();
    }
    return sd.ok ? (int)sd.key : -1;
}

// ---------------------------------------------------------------------------
// Producer warp (one elected lane)
// ---------------------------------------------------------------------------
template <int DT>
__device__ void producer(const KParams& P, const Smem& s) {
    constexpr int ESZ = Elem<DT>::SIZE;
    constexpr int64_t TB = (int64_t)TILE_ELEMS * ESZ;
    volatile int* abort = &s.ctl->abort;
    const uint32_t ns = (uint32_t)P.nstage;
    uint32_t it = 0;
    for (int r = blockIdx.x; r < P.batch; r += gridDim.x) {
        const RowGeom g = row_geom<ESZ>(P, r);
        for (int t = 0; t < g.ntiles; ++t, ++it) {
            const uint32_t st = it % ns, ph = (it / ns) & 1u;
            if (!mbar_wait(&s.empty[st], ph ^ 1u, abort)) {
                *abort = 1;
                // let copies already issued land before the block can exit
                const uint32_t first = it > ns ? it - ns : 0u;
                for (uint32_t j = first; j < it; ++j) {
                    const uint64_t t0 = globaltimer_ns();
                    while (!mbar_test(&s.full[j % ns], (j / ns) & 1u))
                        if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) break;
                }
                return;
            }
            const int64_t off = (int64_t)t * TB;
            const uint32_t bytes = (uint32_t)((g.interior_bytes - off) < TB ? (g.interior_bytes - off) : TB);
            mbar_arrive_expect_tx(&s.full[st], bytes);
            bulk_g2s(s.ring + (int64_t)st * TB, g.interior + off, bytes, &s.full[st]);
        }
    }
}

// ---------------------------------------------------------------------------
// Consumer warps
// ---------------------------------------------------------------------------
template <int DT>
__device__ void consumer(const KParams& P, const Smem& s, const int tid) {
    using E = Elem<DT>;
    constexpr int ESZ = E::SIZE, VEC = E::VEC;
    constexpr int64_t TB = (int64_t)TILE_ELEMS * ESZ;
    constexpr int CPT = (int)(TB / 16 / NCT);
    const int lane = tid & 31, warp = tid >> 5;
    RowCtl* ctl = s.ctl;
    volatile int* abort = &ctl->abort;
    const uint32_t ns = (uint32_t)P.nstage;
    const float scale = __uint_as_float((uint32_t)(127 + P.mass_shift) << 23);  // 2^S
    uint32_t it = 0;
    for (int r = blockIdx.x; r < P.batch; r += gridDim.x) {
        const RowParams p = row_params(P, r);
        const RowGeom g = row_geom<ESZ>(P, r);
        if (tid == 0) {
            ctl->n = 0; ctl->hikey = 0; ctl->xmin = -INFINITY;
            ctl->cand_on = p.cand ? 1 : 0; ctl->status = p.bad; ctl->general = 0;
        }
        csync();
        if (p.pen) history_prologue(P, s, p, r, tid);
        Stream st;
        st.tmax = -INFINITY; st.zm = -1e30f; st.zmc = st.zm * p.c; st.z = 0.0f;
        st.xmin = -INFINITY; st.cand = p.cand;
        const uint8_t* rowp = reinterpret_cast<const uint8_t*>(P.logits) + (int64_t)r * P.row_stride * ESZ;
        // ragged head/tail columns (at most 2*(VEC-1)), one per lane of warp 0
        if (warp == 0) {
            const int nh = g.head, nt = P.vocab - g.tail0;
            const bool valid = lane < nh + nt;
            const int c = lane < nh ? lane : g.tail0 + (lane - nh);
            float x[1] = {-INFINITY};
            if (valid) {
                x[0] = E::load(rowp, c);
                if (p.pen && (hist_bits(s, P.nwords, c, 1) & 1u)) x[0] = penalize(p, s, c, x[0]);
            }
            process<1>(p, s, st, x, valid ? c : 0, valid ? 1u : 0u, lane);
        }
        // streamed interior
        for (int t = 0; t < g.ntiles; ++t, ++it) {
            const uint32_t sidx = it % ns, ph = (it / ns) & 1u;
            const bool ok = mbar_wait(&s.full[sidx], ph, abort);
            if (!ok) *abort = 1;
            const uint8_t* tile = s.ring + (int64_t)sidx * TB;
            const int64_t rem = g.interior_bytes - (int64_t)t * TB;
            const int nch = (int)((rem < TB ? rem : TB) / 16);
#pragma unroll
            for (int j = 0; j < CPT; ++j) {
                const int ch = tid + j * NCT;
                const bool valid = ok && ch < nch;
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                if (valid) v = *reinterpret_cast<const uint4*>(tile + (int64_t)ch * 16);
                float x[VEC];
                E::unpack(v, x);
                const int c0 = g.head + (int)(((int64_t)t * TB + (int64_t)ch * 16) / ESZ);
                if (valid && p.pen) penalize_chunk<VEC>(p, s, P.nwords, c0, x);
                process<VEC>(p, s, st, x, c0, valid ? ((1u << VEC) - 1u) : 0u, lane);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.empty[sidx]);
            if (((t + 1) % CHECK_TILES) == 0 || t == g.ntiles - 1) {
                csync();
                const uint32_t n = ctl->n;
                const bool need = ctl->cand_on && n > (uint32_t)HWM;
                csync();
                if (need) compact(p, s, tid, n);
                st.xmin = ctl->xmin;
                st.cand = ctl->cand_on != 0;
            }
        }
        // uniform snapshot of the abort flag (the producer may set it at any time)
        if (tid == 0) ctl->u32a = (*abort != 0) ? 1u : 0u;
        csync();
        // ---- row statistics ----
        const float M = cons_max_nan(st.tmax, s, tid);
        int64_t out_id = -1;
        int status = ctl->status;
        const bool aborted = ctl->u32a != 0;
        if (aborted) status |= FG_ROW_TIMEOUT;
        double Zq = 0.0;
        if (p.mode == MODE_NUCLEUS && !aborted) {
            double zc = 0.0;
            if (st.z > 0.0f)
                zc = (double)st.z * exp2((double)st.zmc - (double)M * (double)p.c);
            const double Zd = cons_sum_f64(zc, s, tid);
            const float My = ydiv(p, M);
            Zq = Zd * exp((double)M / (double)p.T - (double)My) * (double)scale;
        }
        const bool cand_ok = ctl->cand_on != 0 && ctl->general == 0;
        const uint32_t n = ctl->n;
        csync();
        if (aborted) {
            // nothing trustworthy in this row
        } else if (status & (FG_ROW_BAD_PARAM | FG_ROW_BAD_UNIFORM)) {
            out_id = -1;
        } else if (p.mode == MODE_GREEDY) {
            status |= FG_ROW_GREEDY;
            if (M != M) {
                // torch.argmax: first NaN
                uint32_t best = 0xffffffffu;
                for_row<DT>(P, s, p, r, g, tid, [&](int c, float x) { if (x != x) best = min(best, (uint32_t)c); });
                best = cons_min_u32(best, s, tid);
                out_id = best;
                status |= FG_ROW_GENERAL_PATH;
            } else if (cand_ok) {
                const uint32_t km = fkey(M);
                uint32_t best = 0xffffffffu;
                for (uint32_t i = tid; i < n; i += NCT) if (s.ckey[i] == km) best = min(best, s.cid[i]);
                best = cons_min_u32(best, s, tid);
                out_id = best;
            } else {
                uint32_t best = 0xffffffffu;
                for_row<DT>(P, s, p, r, g, tid, [&](int c, float x) { if (x == M) best = min(best, (uint32_t)c); });
                best = cons_min_u32(best, s, tid);
                out_id = best;
                status |= FG_ROW_GENERAL_PATH;
            }
            if (P.out_probs && out_id >= 0) {
                float* pr = P.out_probs + (int64_t)r * P.vocab;
                for (int c = tid; c < P.vocab; c += NCT) pr[c] = (c == (int)out_id) ? 1.0f : 0.0f;
            }
        } else if (M != M) {
            status |= FG_ROW_NAN;
        } else if (M == INFINITY) {
            status |= FG_ROW_POS_INF;
        } else if (M == -INFINITY) {
            status |= FG_ROW_ALL_MASKED;
        } else {
            const float My = ydiv(p, M);
            bool done = false;
            if (cand_ok && p.mode != MODE_FULL) {
                // candidates -> y-keys and masses
                for (uint32_t i = tid; i < n; i += NCT) s.ckey[i] = fkey(ydiv(p, funkey(s.ckey[i])));
                csync();
                uint32_t ykK = 0;
                bool topk = false;
                if (p.mode == MODE_TOPK) {
                    SelOut so = block_select<true, true>(
                        [&](auto&& f) { for (uint32_t i = tid; i < n; i += NCT) f(s.ckey[i], 1ull); },
                        (uint64_t)(p.K - 1), 32, s, tid);
                    topk = true;
                    ykK = so.ok ? so.key : 0u;
                }
                for (uint32_t i = tid; i < n; i += NCT) {
                    const uint32_t yk = s.ckey[i];
                    s.q[i] = (!topk || yk >= ykK) ? mass_q(funkey(yk), My, scale) : 0ull;
                }
                csync();
                bool not_cov = false;
                const int j = decide(P, s, p, r, tid,
                    [&](auto&& f) { for (uint32_t i = tid; i < n; i += NCT) f(s.ckey[i], s.cid[i], s.q[i]); },
                    topk, ykK, p.mode == MODE_NUCLEUS ? Zq : -1.0, &not_cov);
                if (!not_cov) { out_id = j; done = true; }
            }
            if (!done) {
                status |= FG_ROW_GENERAL_PATH;
                auto row_enum = [&](auto&& f) {
                    for_row<DT>(P, s, p, r, g, tid, [&](int c, float x) {
                        const float y = ydiv(p, x);
                        f(fkey(y), (uint32_t)c, mass_q(y, My, scale));
                    });
                };
                uint32_t ykK = 0;
                bool topk = false;
                if (p.mode == MODE_TOPK) {
                    SelOut so = block_select<true, true>(
                        [&](auto&& f) { for_row<DT>(P, s, p, r, g, tid, [&](int c, float x) { f(fkey(ydiv(p, x)), 1ull); }); },
                        (uint64_t)(p.K - 1), 32, s, tid);
                    topk = true;
                    ykK = so.ok ? so.key : 0u;
                }
                bool not_cov = false;
                out_id = decide(P, s, p, r, tid, row_enum, topk, ykK, -1.0, &not_cov);
            }
            if (out_id < 0 && !(status & FG_ROW_ERROR_MASK)) status |= FG_ROW_ALL_MASKED;
        }
        if (tid == 0) {
            P.out_ids[r] = (out_id >= 0) ? out_id + P.vocab_offset : -1;
            if (P.out_status) P.out_status[r] = status;
        }
        csync();
        if (aborted) {
            // the pipeline gave up: report every remaining row of this CTA and leave
            if (tid == 0)
                for (int rr = r + gridDim.x; rr < P.batch; rr += gridDim.x) {
                    P.out_ids[rr] = -1;
                    if (P.out_status) P.out_status[rr] = FG_ROW_TIMEOUT;
                }
            break;
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(NTHREADS, 1) fg_sample_kernel(const KParams P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem s = carve(smem_raw, P);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < P.nstage; ++i) { mbar_init(&s.full[i], 1); mbar_init(&s.empty[i], NCW); }
        s.ctl->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid >= NCT) {
        if (tid == NCT) producer<DT>(P, s);
        return;
    }
    consumer<DT>(P, s, tid);
}

// ---------------------------------------------------------------------------
// Row argmax with torch.argmax semantics (first NaN, else first maximum).
// ---------------------------------------------------------------------------
struct ArgBest { float v; uint32_t i; };
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
