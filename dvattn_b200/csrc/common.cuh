// Shared device helpers for the sm_100a DVAttn kernels: element types, cp.async with
// zero-fill, ldmatrix / mma.sync fragments, the base-2 exponential, and the per-sequence
// visible-length arithmetic that every kernel agrees on.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dvattn_b200.h"

namespace dvb {

constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

// ----------------------------------------------------------------------------------
// element types
// ----------------------------------------------------------------------------------
template <class T> struct Elem;
template <> struct Elem<float> {
    static constexpr int dtype = DVATTN_FLOAT32;
    __device__ __forceinline__ static float to_f(float x) { return x; }
    __device__ __forceinline__ static float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
    static constexpr int dtype = DVATTN_FLOAT16;
    __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
    __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
    // two floats -> one 32-bit register of two halves (lo = a)
    __device__ __forceinline__ static uint32_t pack2(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};
template <> struct Elem<__nv_bfloat16> {
    static constexpr int dtype = DVATTN_BFLOAT16;
    __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
    __device__ __forceinline__ static uint32_t pack2(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

// ----------------------------------------------------------------------------------
// math
// ----------------------------------------------------------------------------------
// 2^x on the SFU (PTX ex2.approx: max relative error 2^-22 over the normal range;
// ex2(-inf) = +0).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ----------------------------------------------------------------------------------
// cp.async (16 B, L2-only) with zero fill: copies `src_bytes` (0 or 16) bytes and fills
// the rest of the 16-byte destination with zeros.  With src_bytes == 0 nothing is read.
// ----------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ----------------------------------------------------------------------------------
// ldmatrix / mma.sync (m16n8k16, fp32 accumulate)
// ----------------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

template <class T> struct Mma;
template <> struct Mma<__half> {
    __device__ __forceinline__ static void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <> struct Mma<__nv_bfloat16> {
    __device__ __forceinline__ static void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

// Row of `row_bytes` (a multiple of 128) split into 16-byte chunks; chunk c of row r is
// stored at chunk c ^ (r & 7) so that the 8 rows an ldmatrix phase reads hit 8
// different bank groups.
__device__ __forceinline__ uint32_t swz(int row, int chunk, int row_bytes) {
    return static_cast<uint32_t>(row * row_bytes + ((chunk ^ (row & 7)) << 4));
}

// Four consecutive output values of type T in one 8-byte (16-bit T) or 16-byte store.
template <class T> __device__ __forceinline__ void store_quad(T* dst, float a, float b, float c, float d) {
    uint2 pk;
    pk.x = Elem<T>::pack2(a, b);
    pk.y = Elem<T>::pack2(c, d);
    *reinterpret_cast<uint2*>(dst) = pk;
}
template <> __device__ __forceinline__ void store_quad<float>(float* dst, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
}

// ----------------------------------------------------------------------------------
// mbarriers, TMA (non-multicast tiled loads), named barriers, proxy fences
// ----------------------------------------------------------------------------------
// Every wait is bounded: after kWaitNs of polling it gives up and reports failure, so a
// logic error (e.g. a transaction-byte mismatch) ends the kernel with an error flag
// instead of hanging the GPU.
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking test of the phase with `parity`.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase with `parity` to complete; false after kWaitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kWaitNs) return false;
    }
}
// 3-D tiled TMA load (no multicast) completing on an mbarrier; coordinates innermost first.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* map, int x, int y, int z, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* map, int x, int y, int z, int w, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const void* map, int x, int y, int z, int w, int v,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
        "%6}], [%7];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// OR of `pred` over the `n` threads of named barrier `id` (also a barrier).
__device__ __forceinline__ bool named_bar_or(int id, int n, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

// ----------------------------------------------------------------------------------
// Visible keys of one turn for one query: l < L_f and l <= loc (the mask `kp > qp` of
// python/dvattn/attention.py:48-54; negative loc means the turn is skipped,
// src/kernels/varlen_paged_kernel_v21.cuh:76-80).  Positions past the block table
// (max_blocks * block_size) are never visible: the reference would read past the
// table there.
// ----------------------------------------------------------------------------------
__device__ __forceinline__ int visible_len(int L, int loc) {
    int v = min(L, loc + 1);
    return v > 0 ? v : 0;
}

// ----------------------------------------------------------------------------------
// The model's default rotary embedding at one position (HF rotary module): inv_freq_j =
// 1 / base^(2j / R) in f32 (or the module's own table), freq = inv_freq_j * pos (one
// rounding), cos/sin times attention_scaling, returned in the model dtype (round_dtype,
// DVATTN_*) and widened to f32.  Shared by the view builder and the rope-table kernel so
// both give the same bits.
// ----------------------------------------------------------------------------------
__device__ __forceinline__ void rotary_cos_sin(const float* inv_freq, float base, int R, int j, float pos,
                                               float scaling, int round_dtype, float& c, float& s) {
    const float inv = inv_freq ? __ldg(inv_freq + j) : 1.0f / powf(base, (float)(2 * j) / (float)R);
    const float ang = __fmul_rn(inv, pos);
    sincosf(ang, &s, &c);  // one argument reduction for both
    c *= scaling;
    s *= scaling;
    if (round_dtype == DVATTN_BFLOAT16) {
        c = Elem<__nv_bfloat16>::to_f(Elem<__nv_bfloat16>::from_f(c));
        s = Elem<__nv_bfloat16>::to_f(Elem<__nv_bfloat16>::from_f(s));
    } else if (round_dtype == DVATTN_FLOAT16) {
        c = Elem<__half>::to_f(Elem<__half>::from_f(c));
        s = Elem<__half>::to_f(Elem<__half>::from_f(s));
    }
}

}  // namespace dvb
