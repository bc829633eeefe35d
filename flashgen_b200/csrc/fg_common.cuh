// fg_common.cuh — device helpers shared by the sm_100a sampling kernels.
//
// Order-preserving float keys, exact fp32 division, element loads for the
// three logits dtypes, mbarrier / bulk-copy (TMA) wrappers with bounded waits,
// and block-level reductions over a named barrier.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "../../include/flashgen_sampler.h"

namespace fg {

// ---------------------------------------------------------------------------
// Order-preserving keys: key(a) < key(b)  <=>  a < b for non-NaN floats.
// -0.0 is folded onto +0.0 first so that equal values have equal keys, the
// way torch compares them (sampler.py:154 `logit < threshold`).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t fkey(float x) {
    uint32_t u = __float_as_uint(x + 0.0f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float funkey(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}
constexpr uint32_t KEY_NEG_INF = 0x007fffffu;  // fkey(-inf)

// ---------------------------------------------------------------------------
// Correctly rounded x / d for fp32 using a correctly rounded reciprocal r of d
// and one Markstein correction step (P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. R&D 34(1), 1990):
// q0 = x*r; rem = fma(-q0, d, x) (exact); q = fma(rem, r, q0).
// Valid when no intermediate overflows or underflows; outside that range the
// IEEE division intrinsic is used. Tested bit-exact against __fdiv_rn.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float div_rn(float x, float d, float r) {
    float q0 = x * r;
    float rem = __fmaf_rn(-q0, d, x);
    float q = __fmaf_rn(rem, r, q0);
    float ax = fabsf(x);
    if (!(ax >= 0x1p-100f && ax <= 0x1p100f)) q = __fdiv_rn(x, d);  // 0, tiny, huge, inf, NaN
    return q;
}

// ---------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<FG_DTYPE_F32> {
    static constexpr int SIZE = 4;
    static constexpr int VEC = 4;   // elements per 16-byte chunk
    __device__ __forceinline__ static float load(const void* p, int64_t i) {
        return __ldg(reinterpret_cast<const float*>(p) + i);
    }
    __device__ __forceinline__ static void unpack(const uint4& v, float (&x)[4]) {
        x[0] = __uint_as_float(v.x); x[1] = __uint_as_float(v.y);
        x[2] = __uint_as_float(v.z); x[3] = __uint_as_float(v.w);
    }
    __device__ __forceinline__ static void store(void* p, int64_t i, float v) {
        reinterpret_cast<float*>(p)[i] = v;
    }
};
template <> struct Elem<FG_DTYPE_F16> {
    static constexpr int SIZE = 2;
    static constexpr int VEC = 8;
    __device__ __forceinline__ static float load(const void* p, int64_t i) {
        return __half2float(__ldg(reinterpret_cast<const __half*>(p) + i));
    }
    __device__ __forceinline__ static void unpack(const uint4& v, float (&x)[8]) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
            float2 f = __half22float2(h);
            x[2 * i] = f.x; x[2 * i + 1] = f.y;
        }
    }
    __device__ __forceinline__ static void store(void* p, int64_t i, float v) {
        reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    }
};
template <> struct Elem<FG_DTYPE_BF16> {
    static constexpr int SIZE = 2;
    static constexpr int VEC = 8;
    __device__ __forceinline__ static float load(const void* p, int64_t i) {
        uint16_t b = __ldg(reinterpret_cast<const unsigned short*>(p) + i);
        return __uint_as_float(uint32_t(b) << 16);
    }
    __device__ __forceinline__ static void unpack(const uint4& v, float (&x)[8]) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            x[2 * i] = __uint_as_float(w[i] << 16);
            x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    __device__ __forceinline__ static void store(void* p, int64_t i, float v) {
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    }
};

// max that propagates NaN (PTX max.NaN, sm_80+)
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

// ---------------------------------------------------------------------------
// Time source for bounded waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;  // 1 s: far above any legitimate wait

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (sm_90+ PTX; used here on sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Wait for phase `parity` of `bar` to complete. Gives up after WAIT_LIMIT_NS or
// as soon as *abort is set; returns false in that case.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_test(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_test(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) return false;
        }
    }
}
// ---- 32-bit shared-window addresses (the streaming loop keeps no 64-bit
//      pointers live: its addresses are a symbol plus grid-constant offsets)
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ void sts_u32(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" :: "r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atoms_add_u32(uint32_t a, uint32_t v) {
    uint32_t o;
    asm volatile("atom.shared.add.u32 %0, [%1], %2;" : "=r"(o) : "r"(a), "r"(v) : "memory");
    return o;
}
__device__ __forceinline__ bool mbar_test_a(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ void mbar_arrive_a(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" :: "r"(bar) : "memory");
}
// Shared-memory atomics on generic pointers into the dynamic shared memory.
// The pointers come from an opaque base, so a plain atomicAdd would compile to
// a generic atomic, which serialises far more under contention than the
// shared-window form used here.
__device__ __forceinline__ uint32_t atoms_add(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.shared.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(smem_u32(p)), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void reds_add(uint32_t* p, uint32_t v) {
    asm volatile("red.shared.add.u32 [%0], %1;" :: "r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atoms_or(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.shared.or.b32 %0, [%1], %2;" : "=r"(old) : "r"(smem_u32(p)), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void reds_or(uint32_t* p, uint32_t v) {
    asm volatile("red.shared.or.b32 [%0], %1;" :: "r"(smem_u32(p)), "r"(v) : "memory");
}

// mbar_wait on a shared-window address; the abort flag is the int at `abort_a`.
__device__ __forceinline__ bool mbar_wait_a(uint32_t bar, uint32_t parity, uint32_t abort_a) {
    if (mbar_test_a(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_test_a(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            if (lds_u32(abort_a) != 0u) return false;
            if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) return false;
        }
    }
}

// Wait for phase `parity` of `bar` for at most `limit_ns`; returns false on expiry.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_test(bar, parity))
        if (globaltimer_ns() - t0 > limit_ns) return false;
    return true;
}
// 1-D bulk copy global -> shared, completion counted on `bar` (complete_tx).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Same copy with an L2 cache policy (createpolicy) attached to the reads.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy) : "memory");
}
// L2 policy that keeps the lines it fills ahead of normal lines.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// Return the 128-byte L2 line holding `p` to the normal eviction priority.
__device__ __forceinline__ void l2_evict_normal(const void* p) {
    asm volatile("applypriority.global.L2::evict_normal [%0], 128;" :: "l"(p) : "memory");
}

// Named barrier over the first `nthreads` threads of the block (id != 0).
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t shfl_u64(uint64_t v, int src) {
    uint32_t lo = __shfl_sync(0xffffffffu, uint32_t(v), src);
    uint32_t hi = __shfl_sync(0xffffffffu, uint32_t(v >> 32), src);
    return (uint64_t(hi) << 32) | lo;
}
__device__ __forceinline__ uint64_t shfl_up_u64(uint64_t v, int d) {
    uint32_t lo = __shfl_up_sync(0xffffffffu, uint32_t(v), d);
    uint32_t hi = __shfl_up_sync(0xffffffffu, uint32_t(v >> 32), d);
    return (uint64_t(hi) << 32) | lo;
}
__device__ __forceinline__ uint64_t warp_incl_scan_u64(uint64_t v, int lane) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        uint64_t o = shfl_up_u64(v, d);
        if (lane >= d) v += o;
    }
    return v;
}
__device__ __forceinline__ uint32_t warp_incl_scan_u32(uint32_t v, int lane) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        uint32_t o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += o;
    }
    return v;
}

}  // namespace fg
