// forward.cu -- the rest of TinyLlama's forward pass on the device: the
// matrix-vector products of every GGUF weight format (fused with RMSNorm in
// front and a residual add or SwiGLU behind), the embedding lookup and
// greedy sampling.
//
// Reference semantics (src/ops.cpp): matmul() ops.cpp:959-981 with the
// per-format paths F32 ops.cpp:251-262, F16 342-356, Q8_0 442-473, Q4_0
// 616-655, Q6_K 882-948; rmsnorm() ops.cpp:1040-1054; silu() 1107-1113,
// elementwise_mul() 1129-1146, vec_add() 1165-1184, ffn_swiglu() 1535-1564;
// sample_argmax() 1587-1597; embed_token() forward.cpp:35-60.
//
// Design (B200): a decode step reads every weight once, so each product is
// HBM-bound byte work.  The weights are read in place, in the reference's
// GGUF block layout (no repacking: the pointers a GGUF loader hands out
// work unchanged).  One CTA (8 warps) owns a tile of consecutive rows; each
// warp computes whole rows, its lanes splitting a row's blocks (Q4_0/Q8_0:
// 4 lanes per 32-weight block; Q6_K: lane = position l of the 256-weight
// super-block; F16/F32: 16-byte vectors), and a warp shuffle reduces the
// row.  The input vector sits in shared memory, normalised on the way in
// when an RMSNorm precedes the product.  Every kernel is launched as a
// programmatic dependent of the previous one: its CTAs issue a bulk L2
// prefetch of their weight rows (weights are never written by a kernel) and
// only then wait for the previous kernel, so the weight stream of one
// product overlaps the tail of the one before.
#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace tle {

namespace {

constexpr int GT = 256;        // threads per GEMV CTA
constexpr int GW = GT / 32;    // warps per GEMV CTA

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
// 4-bit value n (0..15) minus 8, and an int8 stored as a byte, as floats:
// 2^23 + v has v in its low mantissa bits, so one OR and one subtract do the
// conversion exactly.
__device__ __forceinline__ float nib_m8(uint32_t q, int shift) {
    return __int_as_float(0x4B000000u | ((q >> shift) & 15u)) - 8388616.0f;
}
__device__ __forceinline__ float s8f(uint32_t q, int shift) {
    return __int_as_float(0x4B000000u | (((q >> shift) & 0xFFu) ^ 0x80u)) - 8388736.0f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Per-lane partial dot product of one weight row (GGUF layout) with xs.
// The row is in shared memory (a TMA-staged tile) or in global memory;
// plain loads serve both (the compiler sees which space a pointer is in).
template <int T>
__device__ __forceinline__ float row_dot(const uint8_t* row, const float* xs, int cols, int lane);

__device__ __forceinline__ uint32_t ld16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// F32 (ops.cpp:251-262): 4 consecutive weights per lane (one per lane
// when rows are not 16-byte multiples).
template <>
__device__ __forceinline__ float row_dot<kWF32>(const uint8_t* row, const float* xs, int cols, int lane) {
    float acc = 0.f;
    if (cols & 3) {
        const float* w = reinterpret_cast<const float*>(row);
        for (int c = lane; c < cols; c += 32) acc = fmaf(w[c], xs[c], acc);
        return acc;
    }
    const float4* w = reinterpret_cast<const float4*>(row);
#pragma unroll 4
    for (int c = lane; c < cols / 4; c += 32) {
        const float4 a = w[c];
        const float4 x = *reinterpret_cast<const float4*>(xs + 4 * c);
        acc = fmaf(a.x, x.x, acc);
        acc = fmaf(a.y, x.y, acc);
        acc = fmaf(a.z, x.z, acc);
        acc = fmaf(a.w, x.w, acc);
    }
    return acc;
}

// F16 (ops.cpp:342-356): 8 consecutive weights per lane (one per lane
// when rows are not 16-byte multiples).
template <>
__device__ __forceinline__ float row_dot<kWF16>(const uint8_t* row, const float* xs, int cols, int lane) {
    float acc = 0.f;
    if (cols & 7) {
        const uint16_t* w = reinterpret_cast<const uint16_t*>(row);
        for (int c = lane; c < cols; c += 32) acc = fmaf(h2f(w[c]), xs[c], acc);
        return acc;
    }
    const uint4* w = reinterpret_cast<const uint4*>(row);
#pragma unroll 4
    for (int c = lane; c < cols / 8; c += 32) {
        const uint4 a = w[c];
        const float4 x0 = *reinterpret_cast<const float4*>(xs + 8 * c);
        const float4 x1 = *reinterpret_cast<const float4*>(xs + 8 * c + 4);
        acc = fmaf(h2f(a.x & 0xFFFFu), x0.x, acc);
        acc = fmaf(h2f(a.x >> 16), x0.y, acc);
        acc = fmaf(h2f(a.y & 0xFFFFu), x0.z, acc);
        acc = fmaf(h2f(a.y >> 16), x0.w, acc);
        acc = fmaf(h2f(a.z & 0xFFFFu), x1.x, acc);
        acc = fmaf(h2f(a.z >> 16), x1.y, acc);
        acc = fmaf(h2f(a.w & 0xFFFFu), x1.z, acc);
        acc = fmaf(h2f(a.w >> 16), x1.w, acc);
    }
    return acc;
}

// Q4_0 (ops.cpp:616-655): block = fp16 d + 16 bytes; byte j holds element
// j (low nibble) and j + 16 (high nibble).  Lane t = lane & 3 of a block
// takes bytes 4t..4t+3: elements 4t..4t+3 and 16+4t..16+4t+3.  Its 8-term
// block partial is scaled by d like the reference's block sum.
template <>
__device__ __forceinline__ float row_dot<kWQ4_0>(const uint8_t* row, const float* xs, int cols, int lane) {
    const int nb = cols >> 5;
    const int t = lane & 3;
    float acc = 0.f;
#pragma unroll 4
    for (int b = lane >> 2; b < nb; b += 8) {
        const uint8_t* blk = row + 18 * b;
        const float d = h2f(static_cast<uint16_t>(ld16(blk)));
        const uint32_t q = ld16(blk + 2 + 4 * t) | (ld16(blk + 4 + 4 * t) << 16);
        const float4 xl = *reinterpret_cast<const float4*>(xs + 32 * b + 4 * t);
        const float4 xh = *reinterpret_cast<const float4*>(xs + 32 * b + 16 + 4 * t);
        float s = nib_m8(q, 0) * xl.x;
        s = fmaf(nib_m8(q, 4), xh.x, s);
        s = fmaf(nib_m8(q, 8), xl.y, s);
        s = fmaf(nib_m8(q, 12), xh.y, s);
        s = fmaf(nib_m8(q, 16), xl.z, s);
        s = fmaf(nib_m8(q, 20), xh.z, s);
        s = fmaf(nib_m8(q, 24), xl.w, s);
        s = fmaf(nib_m8(q, 28), xh.w, s);
        acc = fmaf(d, s, acc);
    }
    return acc;
}

// Q8_0 (ops.cpp:442-473): block = fp16 d + 32 int8.  Lane t takes elements
// 8t..8t+7 of each of its blocks.
template <>
__device__ __forceinline__ float row_dot<kWQ8_0>(const uint8_t* row, const float* xs, int cols, int lane) {
    const int nb = cols >> 5;
    const int t = lane & 3;
    float acc = 0.f;
#pragma unroll 4
    for (int b = lane >> 2; b < nb; b += 8) {
        const uint8_t* blk = row + 34 * b;
        const float d = h2f(static_cast<uint16_t>(ld16(blk)));
        const uint8_t* qs = blk + 2 + 8 * t;
        const uint32_t q0 = ld16(qs) | (ld16(qs + 2) << 16);
        const uint32_t q1 = ld16(qs + 4) | (ld16(qs + 6) << 16);
        const float4 x0 = *reinterpret_cast<const float4*>(xs + 32 * b + 8 * t);
        const float4 x1 = *reinterpret_cast<const float4*>(xs + 32 * b + 8 * t + 4);
        float s = s8f(q0, 0) * x0.x;
        s = fmaf(s8f(q0, 8), x0.y, s);
        s = fmaf(s8f(q0, 16), x0.z, s);
        s = fmaf(s8f(q0, 24), x0.w, s);
        s = fmaf(s8f(q1, 0), x1.x, s);
        s = fmaf(s8f(q1, 8), x1.y, s);
        s = fmaf(s8f(q1, 16), x1.z, s);
        s = fmaf(s8f(q1, 24), x1.w, s);
        acc = fmaf(d, s, acc);
    }
    return acc;
}

// Q6_K (ops.cpp:882-948): super-block of 256 = ql[128], qh[64], int8
// scales[16], fp16 d.  Lane l takes position l of both halves: the four
// 6-bit values built from ql[l], ql[l+32] and qh[l] of each half.
template <>
__device__ __forceinline__ float row_dot<kWQ6_K>(const uint8_t* row, const float* xs, int cols, int lane) {
    const int nb = cols >> 8;
    const int is = lane >> 4;
    float acc = 0.f;
    for (int b = 0; b < nb; ++b) {
        const uint8_t* blk = row + 210 * b;
        const float d = h2f(static_cast<uint16_t>(ld16(blk + 208)));
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t l0 = blk[64 * h + lane];
            const uint32_t l1 = blk[64 * h + lane + 32];
            const uint32_t hh = blk[128 + 32 * h + lane];
            const float* X = xs + 256 * b + 128 * h;
            const int q1 = static_cast<int>((l0 & 15u) | ((hh & 3u) << 4)) - 32;
            const int q2 = static_cast<int>((l1 & 15u) | (((hh >> 2) & 3u) << 4)) - 32;
            const int q3 = static_cast<int>((l0 >> 4) | (((hh >> 4) & 3u) << 4)) - 32;
            const int q4 = static_cast<int>((l1 >> 4) | (((hh >> 6) & 3u) << 4)) - 32;
            const int8_t* S = sc + 8 * h + is;
            acc = fmaf(d * static_cast<float>(S[0]) * static_cast<float>(q1), X[lane], acc);
            acc = fmaf(d * static_cast<float>(S[2]) * static_cast<float>(q2), X[lane + 32], acc);
            acc = fmaf(d * static_cast<float>(S[4]) * static_cast<float>(q3), X[lane + 64], acc);
            acc = fmaf(d * static_cast<float>(S[6]) * static_cast<float>(q4), X[lane + 96], acc);
        }
    }
    return acc;
}

__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 up2(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// Nibble values of bytes j, k of w (each byte holding one 4-bit value) as the
// float pair (n_j - 8, n_k - 8): the byte permute builds 2^23 + n exactly,
// one packed subtract removes 2^23 + 8.
__device__ __forceinline__ uint64_t nib_pair(uint32_t w, int j, int k) {
    const float a = __int_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | j));
    const float b = __int_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | k));
    return add2(pk2(a, b), pk2(-8388616.0f, -8388616.0f));
}

// Q4_0 rows from shared memory, R rows at once: each lane's slice of the
// input vector is read once per block and used for all R rows (reading it
// per row made the kernel shared-memory bound).  Lane t = lane & 3 of a
// block takes bytes 4t..4t+3 (elements 4t..4t+3 low nibbles, 16+4t..
// high nibbles); products as packed f32x2 FMAs, the 8-term block partial
// scaled by d as the reference does per block.
template <int R>
__device__ __forceinline__ void rows_dot_q4(const uint8_t* const (&rows)[R], const float* xs, int b_lo,
                                            int b_hi, int lane, float (&acc)[R]) {
    const int t = lane & 3;
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = 0.f;
#pragma unroll 2
    for (int b = b_lo + (lane >> 2); b < b_hi; b += 8) {
        const float4 xl = *reinterpret_cast<const float4*>(xs + 32 * b + 4 * t);
        const float4 xh = *reinterpret_cast<const float4*>(xs + 32 * b + 16 + 4 * t);
        const uint64_t x01 = pk2(xl.x, xl.y), x23 = pk2(xl.z, xl.w);
        const uint64_t h01 = pk2(xh.x, xh.y), h23 = pk2(xh.z, xh.w);
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const uint8_t* blk = rows[i] + 18 * b;
            const float d = h2f(static_cast<uint16_t>(ld16(blk)));
            const uint32_t q = ld16(blk + 2 + 4 * t) | (ld16(blk + 4 + 4 * t) << 16);
            const uint32_t lo = q & 0x0F0F0F0Fu, hi = (q >> 4) & 0x0F0F0F0Fu;
            uint64_t s2 = fma2(nib_pair(lo, 0, 1), x01, 0ull);
            s2 = fma2(nib_pair(lo, 2, 3), x23, s2);
            s2 = fma2(nib_pair(hi, 0, 1), h01, s2);
            s2 = fma2(nib_pair(hi, 2, 3), h23, s2);
            const float2 s = up2(s2);
            acc[i] = fmaf(d, s.x + s.y, acc[i]);
        }
    }
}

// Bulk prefetch into L2 of [p, p + bytes), trimmed inward to 16-byte
// boundaries (a hint: the trimmed edges are simply not prefetched).
__device__ __forceinline__ void prefetch_l2(const uint8_t* p, size_t bytes) {
    uintptr_t a = (reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15);
    uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes) & ~uintptr_t(15);
    while (a < e) {
        const uintptr_t left = e - a;
        const uint32_t n = static_cast<uint32_t>(left < (uintptr_t(1) << 20) ? left : (uintptr_t(1) << 20));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
        a += n;
    }
}

// Stages the input vector into xs with ordered L2 loads (it is the previous
// kernel's output), D 16-byte loads in flight per thread (NT threads) before
// any is stored; returns this thread's share of sum(x^2).
template <int NT = GT, int D = 8>
__device__ __forceinline__ float stage_x(float* xs, const float* x, int cols, int tid) {
    float ss = 0.f;
    if ((cols & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const int n4 = cols >> 2;
        for (int base = tid; base < n4; base += NT * D) {
            float4 v[D];
#pragma unroll
            for (int j = 0; j < D; ++j) {
                const int i = base + j * NT;
                if (i < n4) v[j] = ld_cg4(reinterpret_cast<const float4*>(x) + i);
            }
#pragma unroll
            for (int j = 0; j < D; ++j) {
                const int i = base + j * NT;
                if (i < n4) {
                    reinterpret_cast<float4*>(xs)[i] = v[j];
                    ss = fmaf(v[j].x, v[j].x, ss);
                    ss = fmaf(v[j].y, v[j].y, ss);
                    ss = fmaf(v[j].z, v[j].z, ss);
                    ss = fmaf(v[j].w, v[j].w, ss);
                }
            }
        }
    } else {
        for (int base = tid; base < cols; base += NT * D) {
            float v[D];
#pragma unroll
            for (int j = 0; j < D; ++j) {
                const int i = base + j * NT;
                if (i < cols) v[j] = ld_cg(x + i);
            }
#pragma unroll
            for (int j = 0; j < D; ++j) {
                const int i = base + j * NT;
                if (i < cols) {
                    xs[i] = v[j];
                    ss = fmaf(v[j], v[j], ss);
                }
            }
        }
    }
    return ss;
}

// One launch: rows of up to three matrices that share the input vector
// (q, k and v of a layer), or gate and up rows for SwiGLU.  TMA: the CTA's
// rows are one contiguous span of the weights; a single 1-D bulk copy (two
// for SwiGLU) brings them into shared memory, issued before the wait on
// the previous kernel.  Otherwise (rows not 16-byte multiples) the rows are
// read from global memory after an L2 prefetch.
template <int T, int EPI, bool TMA>
__global__ void __launch_bounds__(GT) gemv_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(16) unsigned char gsm[];
    __shared__ float red[GW];
    __shared__ float part[2][GW][4];   // Q4_0 path: per column chunk, per row group partial sums
    __shared__ __align__(8) uint64_t wbar;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rows_per_cta = a.rpc;
    float* xs = reinterpret_cast<float*>(gsm);
    unsigned char* tile = gsm + a.xs_bytes;
    unsigned char* tile2 = tile + a.tile_bytes;

    int s = 0;
    while (s + 1 < a.n_seg && static_cast<int>(blockIdx.x) >= a.seg[s + 1].tile0) ++s;
    const GemvSeg& seg = a.seg[s];
    const int r0 = (static_cast<int>(blockIdx.x) - seg.tile0) * rows_per_cta;
    const int r1 = min(r0 + rows_per_cta, seg.rows);
    const size_t off0 = static_cast<size_t>(r0) * a.row_bytes;
    const uint32_t span = static_cast<uint32_t>(r1 - r0) * static_cast<uint32_t>(a.row_bytes);

    // Weights are never written by a kernel: fetch them before the wait.
    if (tid == 0) {
        if (TMA) {
            mbar_init(&wbar, 1);
            fence_barrier_init();
            mbar_arrive_expect_tx(&wbar, (EPI == kEpiSwiGLU ? 2u : 1u) * span);
            bulk_g2s_plain(tile, seg.W + off0, span, &wbar);
            if (EPI == kEpiSwiGLU) bulk_g2s_plain(tile2, a.W2 + off0, span, &wbar);
        } else {
            prefetch_l2(seg.W + off0, span);
            if (EPI == kEpiSwiGLU) prefetch_l2(a.W2 + off0, span);
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // The input vector, normalised (rmsnorm, ops.cpp:1040-1054: x * rms *
    // weight with rms = 1 / sqrt(mean(x^2) + eps)) when a norm weight is
    // given.
    float ss = stage_x(xs, a.x, a.cols, tid);
    if (a.norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            float v = lane < GW ? red[lane] : 0.f;
            v = warp_sum(v);
            if (lane == 0) red[0] = 1.0f / sqrtf(v / static_cast<float>(a.cols) + a.eps);
        }
        __syncthreads();
        const float rms = red[0];
        for (int i = tid; i < a.cols; i += GT) xs[i] = xs[i] * rms * a.norm_w[i];
    }
    __syncthreads();
    bool ok = true;
    if (TMA) {
        ok = __all_sync(0xffffffffu, mbar_wait(&wbar, 0));
        if (!ok) {
            if (lane == 0) record_error(a.err, kErrWaitFull);
            // the copy may still be in flight: wait once more before the
            // CTA (and its shared memory) goes away
            mbar_wait(&wbar, 0);
        }
    }

    if constexpr (T == kWQ4_0 && TMA) {
        // Warps = (GW / ks) row groups of 4 rows x ks column chunks; SwiGLU
        // runs a group's 4 gate and 4 up rows together (8 rows sharing the
        // input reads).  Chunk partials are summed in chunk order.
        constexpr int R = (EPI == kEpiSwiGLU) ? 8 : 4;
        const int ks = a.ks;
        const int g = warp / ks, kc = warp - g * ks;
        const int nb = a.cols >> 5;
        const int chunk = ((nb + ks - 1) / ks + 7) & ~7;
        const int b_lo = kc * chunk, b_hi = min(nb, b_lo + chunk);
        const int rb = r0 + 4 * g;
        float acc[R];
        if (ok && rb < r1) {
            const uint8_t* rp[R];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int rr = min(rb + i, r1 - 1) - r0;   // rows past r1 repeat the last one
                rp[i] = tile + static_cast<size_t>(rr) * a.row_bytes;
                if (EPI == kEpiSwiGLU) rp[i + 4] = tile2 + static_cast<size_t>(rr) * a.row_bytes;
            }
            rows_dot_q4<R>(rp, xs, b_lo, b_hi, lane, acc);
#pragma unroll
            for (int i = 0; i < R; ++i) acc[i] = warp_sum(acc[i]);
            if (lane == 0) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    part[0][warp][i] = acc[i];
                    if (EPI == kEpiSwiGLU) part[1][warp][i] = acc[i + 4];
                }
            }
        }
        __syncthreads();
        if (ok && tid < rows_per_cta) {
            const int gg = tid >> 2, i = tid & 3;
            const int r = r0 + tid;
            if (r < r1) {
                float y = 0.f, u = 0.f;
                for (int c = 0; c < ks; ++c) {
                    y += part[0][gg * ks + c][i];
                    if (EPI == kEpiSwiGLU) u += part[1][gg * ks + c][i];
                }
                if (EPI == kEpiSwiGLU) {
                    // silu(g) * u (ops.cpp:1107-1113 then 1129-1146)
                    seg.out[r] = (y * (1.0f / (1.0f + expf(-y)))) * u;
                } else if (EPI == kEpiAdd) {
                    seg.out[r] = ld_cg(seg.out + r) + y;
                } else {
                    seg.out[r] = y;
                }
            }
        }
    } else {
    for (int k = 0; ok && k < a.rpw; ++k) {
        const int r = r0 + warp * a.rpw + k;
        if (r >= r1) break;
        const uint8_t* wr = TMA ? tile + static_cast<size_t>(r - r0) * a.row_bytes
                                : seg.W + static_cast<size_t>(r) * a.row_bytes;
        const float y = warp_sum(row_dot<T>(wr, xs, a.cols, lane));
        if (EPI == kEpiSwiGLU) {
            const uint8_t* ur = TMA ? tile2 + static_cast<size_t>(r - r0) * a.row_bytes
                                    : a.W2 + static_cast<size_t>(r) * a.row_bytes;
            const float u = warp_sum(row_dot<T>(ur, xs, a.cols, lane));
            // silu(g) * u (ops.cpp:1107-1113 then 1129-1146)
            if (lane == 0) seg.out[r] = (y * (1.0f / (1.0f + expf(-y)))) * u;
        } else if (EPI == kEpiAdd) {
            if (lane == 0) seg.out[r] = ld_cg(seg.out + r) + y;
        } else {
            if (lane == 0) seg.out[r] = y;
        }
    }
    }
}

// embed_token (forward.cpp:35-60): row `token` of the table, as fp32.  A
// token outside [0, n_vocab) is reported (0x106) and gives a zero row.
template <int T>
__global__ void __launch_bounds__(256) embed_kernel(float* __restrict__ x, const uint8_t* __restrict__ table,
                                                     const int32_t* token, int n_vocab, int n_embd,
                                                     uint32_t* err) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int t = ld_cg_s32(token);   // the previous step's sampler may have written it
    const bool ok = t >= 0 && t < n_vocab;
    if (!ok && threadIdx.x == 0 && blockIdx.x == 0) record_error(err, kErrBadToken);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_embd; i += gridDim.x * blockDim.x) {
        float v = 0.f;
        if (ok) {
            const size_t e = static_cast<size_t>(t) * n_embd + i;
            v = (T == kWF16) ? h2f(__ldg(reinterpret_cast<const unsigned short*>(table) + e))
                             : __ldg(reinterpret_cast<const float*>(table) + e);
        }
        x[i] = v;
    }
}

// sample_argmax (ops.cpp:1587-1597): the first index of the maximum under
// '>'.  A NaN never beats the running best, so NaNs after index 0 are
// skipped; a NaN at index 0 makes the answer 0 (nothing compares greater).
__global__ void __launch_bounds__(1024) argmax_kernel(const float* logits, int n, int32_t* out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int base = tid; base < n; base += 1024 * 32) {
        float vs[32];                        // 32 loads in flight (a 32 K vocabulary in one round trip), then the scan
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int i = base + j * 1024;
            vs[j] = i < n ? ld_cg(logits + i) : -INFINITY;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int i = base + j * 1024;
            float v = vs[j];
            if (i >= n) break;
            if (v != v) v = -INFINITY;           // NaN: never the maximum
            if (bi == 0x7fffffff || v > bv) {    // first element of this thread, or strictly greater
                bv = v;
                bi = i;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((tid & 31) == 0) {
        sv[tid >> 5] = bv;
        si[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid < 32) {
        bv = sv[tid];
        bi = si[tid];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (tid == 0) {
            const float v0 = ld_cg(logits);
            *out = (v0 != v0) ? 0 : bi;
        }
    }
}

// sample_temperature / sample_top_p (ops.cpp:1624-1722) with the uniform
// draw r given.  One CTA: the row is scaled by 1/T (when T != 1 and T > 0),
// turned into probabilities (softmax ops.cpp:1072-1091: max, exp, times
// 1/sum) in shared memory and written back over the logits as the
// reference does.  Temperature: thread t owns the contiguous chunk t of the
// row; chunk sums, a block scan, then the owner of the first crossing of r
// walks its chunk in index order (n - 1 if the sum never exceeds r).  Top-p:
// the largest threshold whose tail mass reaches top_p (binary search on
// the float bits), the tokens at or above it (at most kTopPMax, the most
// probable kept when more) bitonic-sorted by (probability descending, index
// ascending), then one thread walks them as the reference walks its
// partially sorted order: cumulative sum to top_p, r scaled by it, first
// running sum above it.
constexpr int kSampleThreads = 1024;
constexpr int kTopPMax = 2048;

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        float w = warp_sum(red[threadIdx.x]);
        if (threadIdx.x == 0) red[0] = w;
    }
    __syncthreads();
    return red[0];
}

template <bool TOP_P>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(float* logits, int n, float temperature,
                                                                float top_p, float r, int32_t* out) {
    extern __shared__ __align__(16) float sp[];     // [n] probabilities, then top-p candidates
    __shared__ float red[32];
    __shared__ int best;
    __shared__ int cnt;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x;
    const bool scale = temperature != 1.0f && temperature > 0.0f;
    const float inv_temp = scale ? 1.0f / temperature : 1.0f;
    float mx = -INFINITY;
    for (int base = tid; base < n; base += kSampleThreads * 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = base + j * kSampleThreads;
            v[j] = i < n ? ld_cg(logits + i) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = base + j * kSampleThreads;
            if (i < n) {
                const float x = scale ? v[j] * inv_temp : v[j];
                sp[i] = x;
                mx = fmaxf(mx, x);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    if (tid < 32) {
        float w = red[tid];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
        if (tid == 0) red[0] = w;
    }
    __syncthreads();
    mx = red[0];
    float sum = 0.f;
    for (int i = tid; i < n; i += kSampleThreads) {
        const float e = expf(sp[i] - mx);
        sp[i] = e;
        sum += e;
    }
    sum = block_sum(sum, red);
    const float inv_sum = 1.0f / sum;
    for (int i = tid; i < n; i += kSampleThreads) {
        const float p = sp[i] * inv_sum;
        sp[i] = p;
        logits[i] = p;
    }
    __syncthreads();

    if (!TOP_P) {
        const int per = (n + kSampleThreads - 1) / kSampleThreads;
        const int c0 = min(n, tid * per), c1 = min(n, c0 + per);
        float cs = 0.f;
        for (int i = c0; i < c1; ++i) cs += sp[i];
        // inclusive block scan of the chunk sums (warp shuffles, then one
        // warp over the warp totals)
        float incl = cs;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, incl, o);
            if ((tid & 31) >= o) incl += y;
        }
        if ((tid & 31) == 31) red[tid >> 5] = incl;
        if (tid == 0) best = n - 1;
        __syncthreads();
        if (tid < 32) {
            float w = red[tid];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, w, o);
                if (tid >= o) w += y;
            }
            red[tid] = w;
        }
        __syncthreads();
        const float prefix = incl - cs + ((tid >> 5) ? red[(tid >> 5) - 1] : 0.f);
        if (c1 > c0 && prefix + cs > r) {
            float running = prefix;
            int found = c1 - 1;
            for (int i = c0; i < c1; ++i) {
                running += sp[i];
                if (running > r) {
                    found = i;
                    break;
                }
            }
            atomicMin(&best, found);
        }
        __syncthreads();
        if (tid == 0) *out = best;
        return;
    }

    // top-p: the largest t (float bits; probabilities are >= 0) whose tail
    // mass sum(p >= t) reaches top_p
    float* cp = sp + ((n + 3) & ~3);
    int* ci = reinterpret_cast<int*>(cp + kTopPMax);
    unsigned lo = 0u, hi = __float_as_uint(1.0f);
    while (lo < hi) {
        const unsigned mid = lo + (hi - lo + 1) / 2;
        const float t = __uint_as_float(mid);
        float m = 0.f;
        for (int i = tid; i < n; i += kSampleThreads)
            if (sp[i] >= t) m += sp[i];
        m = block_sum(m, red);
        if (m >= top_p) lo = mid; else hi = mid - 1;
    }
    // at most kTopPMax candidates: raise the threshold while there are more
    unsigned t_bits = lo;
    for (;;) {
        const float t = __uint_as_float(t_bits);
        float c = 0.f;
        for (int i = tid; i < n; i += kSampleThreads) c += (sp[i] >= t) ? 1.f : 0.f;
        c = block_sum(c, red);
        if (c <= kTopPMax) break;
        unsigned a = t_bits + 1, b = __float_as_uint(1.0f);   // smallest bits with count <= max
        while (a < b) {
            const unsigned mid = a + (b - a) / 2;
            const float tm = __uint_as_float(mid);
            float cm = 0.f;
            for (int i = tid; i < n; i += kSampleThreads) cm += (sp[i] >= tm) ? 1.f : 0.f;
            cm = block_sum(cm, red);
            if (cm <= kTopPMax) b = mid; else a = mid + 1;
        }
        t_bits = a;
    }
    if (tid == 0) cnt = 0;
    __syncthreads();
    const float t = __uint_as_float(t_bits);
    for (int i = tid; i < n; i += kSampleThreads)
        if (sp[i] >= t) {
            const int k = atomicAdd(&cnt, 1);
            if (k < kTopPMax) {
                cp[k] = sp[i];
                ci[k] = i;
            }
        }
    __syncthreads();
    const int m = min(cnt, kTopPMax);
    int P2 = 1;
    while (P2 < m) P2 <<= 1;
    for (int k = m + tid; k < P2; k += kSampleThreads) {
        cp[k] = -1.f;
        ci[k] = 0x7fffffff;
    }
    __syncthreads();
    // bitonic sort: probability descending, then index ascending
    for (int size = 2; size <= P2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int k = tid; k < P2; k += kSampleThreads) {
                const int j = k ^ stride;
                if (j > k) {
                    const bool desc = (k & size) == 0;
                    const float pk = cp[k], pj = cp[j];
                    const int ik = ci[k], ij = ci[j];
                    const bool k_first = pk > pj || (pk == pj && ik < ij);
                    if (desc != k_first) {
                        cp[k] = pj;
                        cp[j] = pk;
                        ci[k] = ij;
                        ci[j] = ik;
                    }
                }
            }
            __syncthreads();
        }
    }
    if (tid == 0) {
        float cumsum = 0.f;
        int cutoff = 0;
        for (int k = 0; k < m; ++k) {
            cumsum += cp[k];
            cutoff = k + 1;
            if (cumsum >= top_p) break;
        }
        const float rr = r * cumsum;
        float running = 0.f;
        int tok = ci[0];
        for (int k = 0; k < cutoff; ++k) {
            running += cp[k];
            if (running > rr) {
                tok = ci[k];
                break;
            }
        }
        *out = tok;
    }
}

// rmsnorm (ops.cpp:1040-1054) as its own launch (one CTA): out may alias x.
__global__ void __launch_bounds__(1024) rmsnorm_kernel(float* out, const float* x, const float* w,
                                                       int n, float eps) {
    __shared__ float red[32];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x;
    float ss = 0.f;
    for (int i = tid; i < n; i += 1024) {
        const float v = ld_cg(x + i);
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
        float v = warp_sum(red[tid]);
        if (tid == 0) red[0] = 1.0f / sqrtf(v / static_cast<float>(n) + eps);
    }
    __syncthreads();
    const float rms = red[0];
    for (int i = tid; i < n; i += 1024) out[i] = ld_cg(x + i) * rms * w[i];
}

// vec_add (ops.cpp:1165-1184): out += x.
__global__ void __launch_bounds__(256) vec_add_kernel(float* out, const float* x, int n) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = ld_cg(out + i) + ld_cg(x + i);
}

// ---- persistent forward of one token (all-Q4_0 layers) ---------------------
// One cooperative launch of one CTA per SM runs every layer of a token:
//   P1 RMSNorm(x) + q/k/v rows   P2 rope + attention + append (row pos)
//   P3 x += Wo attn              P4 RMSNorm(x) + gate/up rows + SwiGLU -> hb
//   P5 x += Wdown hb
// with a grid barrier after each phase (every product reads the whole
// output of the one before).  CTA b owns rows [b R, (b+1) R) of every
// product (R = ceil(rows / grid)); its rows of the products to come are
// bulk-copied (TMA engine, one copy per contiguous span) into one of two shared-memory buffers before the barrier of the phase that
// precedes their use (weights are never written, so the copies run ahead
// freely): Wo at P1, gate/up at P2, Wdown at P4, the next layer's q/k/v at
// P5.  Buffer A holds q/k/v and gate/up, buffer B Wo and Wdown.
//
// Products: a thread takes one (row, unit) pair, a unit being 8 Q4_0 blocks
// (256 weights, 144 bytes = nine 16-byte shared loads), and writes its
// partial; the partials of a row are then summed in unit order.  Adjacent
// threads hold adjacent units of a row: their 16-byte weight loads are 144
// bytes apart (nine chunks, so eight threads cover all banks), and the input
// vector is staged with its 16-byte chunks rotated by the unit index inside
// each block, so eight units' reads of the same input chunk hit distinct
// banks too.  RMSNorm: x * w is
// staged while sum(x^2) is reduced; the row sums are scaled by 1/rms.
//
// Attention (P2) splits the L = pos + 1 rows of each KV head over C = L / 64
// CTAs (rounded up); their cached K/V rows are copied into shared memory at
// P1, so P2 waits only for q, k, v.  Warp w takes query head 8 g + (w & 7)
// over half (w >> 3) of the chunk's rows; the halves are folded in shared
// memory and each CTA writes one (o, max, sum) record per head.  The records
// are folded (chunk order) by every CTA while it stages P3's input.  Every
// read of an activation another CTA wrote goes through L2 (ld.cg), after an
// acquire at the barrier.
constexpr int PT = 512;   // 16 warps
constexpr int PW = PT / 32;
constexpr int PKP = 68;   // padded K/V row of the attention phase (floats)
constexpr int kUnit = 256;            // weights per unit
constexpr int kUnitBytes = 144;       // Q4_0 bytes per unit
constexpr int kRec = 68;              // floats per attention record: o[64], max, sum, 2 pad
constexpr int kAttRows = kPersistAttRows;

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier over gridDim.x CTAs (all resident: cooperative launch).  The
// count only grows within a launch; barrier k waits for (k + 1) * grid
// arrivals.  A wait that gives up (2 s) records 0x108 and the CTA stops
// waiting at later barriers, so the launch always ends.
__device__ __forceinline__ void grid_barrier(uint32_t* ctr, uint32_t target, uint32_t* err, int* failed) {
    __syncthreads();
    if (threadIdx.x == 0 && !*failed) {
        // release: the CTA's writes (ordered before this thread by the
        // barrier above) before the arrival; acquire on the count
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
        if (ld_acquire_u32(ctr) < target) {
            const uint64_t t0 = globaltimer();
            while (ld_acquire_u32(ctr) < target) {
                if (globaltimer() - t0 > kWaitTimeoutNs) {
                    record_error(err, kErrGridWait);
                    *failed = 1;
                    break;
                }
            }
        }
    }
    __syncthreads();
}

__device__ __forceinline__ int cta_rows(int rows, int b, int G, int& r0) {
    const int R = (rows + G - 1) / G;
    r0 = min(rows, b * R);
    return max(0, min(rows, r0 + R) - r0);
}

// Float index of input element f in the staged (rotated) layout: chunk i of
// block k of unit u sits at chunk (i + u) mod 8 of the block.
__device__ __forceinline__ int xs_phys(int f) {
    return (f & ~31) | (((((f >> 2) + (f >> 8)) & 7)) << 2) | (f & 3);
}

// The products read the staged input scaled by 2^100 and each weight as the
// subnormal float n * 2^-149 (one byte permute, exact): a product is then
// n x 2^-49, a normal float for any |x| in [2^-77, 2^27], and the Q4_0
// offset is taken per block, sum((n - 8) x) = sum(n x) - 8 sum(x), with
// 8 sum(x) 2^-49 precomputed here (bs).  Row sums are scaled back by 2^49.
constexpr float kXScale = 0x1p100f;
constexpr float kBlockSumScale = 0x1p-146f;   // 8 * 2^-149
constexpr float kRowScale = 0x1p49f;

// Lanes 8k..8k+7 stage the eight float4 of one 32-input block (i is
// warp-uniform in range): t scaled into xs, the block's 8 sum(x) 2^-49 into
// bs[i / 8].
__device__ __forceinline__ void stage_store(float* xs, float* bs, int i, float4 t) {
    t = make_float4(t.x * kXScale, t.y * kXScale, t.z * kXScale, t.w * kXScale);
    *reinterpret_cast<float4*>(xs + xs_phys(4 * i)) = t;
    float sum = (t.x + t.y) + (t.z + t.w);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if ((i & 7) == 0) bs[i >> 3] = sum * kBlockSumScale;
}

// Stages x (times w when w is given) into xs in the rotated layout, with
// the block sums; returns this thread's share of sum(x^2).  cols % 256 == 0.
__device__ __forceinline__ float stage_rot(float* xs, float* bs, const float* x, const float* w, int cols) {
    float ss = 0.f;
    const int n4 = cols >> 2;
    for (int base = threadIdx.x; base < n4; base += 2 * PT) {
        float4 v[2], g[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = base + j * PT;
            if (i < n4) {
                v[j] = ld_cg4(reinterpret_cast<const float4*>(x) + i);
                if (w) g[j] = __ldg(reinterpret_cast<const float4*>(w) + i);
            }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = base + j * PT;
            if (i < n4) {
                float4 t = v[j];
                ss = fmaf(t.x, t.x, ss);
                ss = fmaf(t.y, t.y, ss);
                ss = fmaf(t.z, t.z, ss);
                ss = fmaf(t.w, t.w, ss);
                if (w) t = make_float4(t.x * g[j].x, t.y * g[j].y, t.z * g[j].z, t.w * g[j].w);
                stage_store(xs, bs, i, t);
            }
        }
    }
    return ss;
}

// The attention output (32 heads x 64) folded from the chunk records, in
// chunk order (max first, then the rescaled sums), staged rotated into xs.
__device__ __forceinline__ void stage_attention(float* xs, float* bs, const float* rec, int n_chunks, int n_embd) {
    for (int i = threadIdx.x; i < (n_embd >> 2); i += PT) {
        const int h = i >> 4, d0 = 4 * (i & 15);
        if (n_chunks <= 8) {   // every record load in flight at once (one L2 round trip)
            float mc[8], lc[8];
            float4 oc[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                mc[c] = -INFINITY;
                lc[c] = 0.f;
                oc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (c < n_chunks) {
                    const float* R = rec + (c * kNHead + h) * kRec;
                    mc[c] = ld_cg(R + kHeadDim);
                    lc[c] = ld_cg(R + kHeadDim + 1);
                    oc[c] = ld_cg4(reinterpret_cast<const float4*>(R + d0));
                }
            }
            float mt = -INFINITY;
#pragma unroll
            for (int c = 0; c < 8; ++c) mt = fmaxf(mt, mc[c]);
            float lt = 0.f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                if (c < n_chunks) {
                    const float f = expf(mc[c] - mt);
                    lt = fmaf(lc[c], f, lt);
                    acc.x = fmaf(oc[c].x, f, acc.x);
                    acc.y = fmaf(oc[c].y, f, acc.y);
                    acc.z = fmaf(oc[c].z, f, acc.z);
                    acc.w = fmaf(oc[c].w, f, acc.w);
                }
            }
            const float inv = 1.0f / lt;
            stage_store(xs, bs, i, make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
            continue;
        }
        float mt = -INFINITY;
        for (int c = 0; c < n_chunks; ++c) mt = fmaxf(mt, ld_cg(rec + (c * kNHead + h) * kRec + kHeadDim));
        float lt = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        int c = 0;
        for (; c + 4 <= n_chunks; c += 4) {
            float mc[4], lc[4];
            float4 oc[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float* R = rec + ((c + u) * kNHead + h) * kRec;
                mc[u] = ld_cg(R + kHeadDim);
                lc[u] = ld_cg(R + kHeadDim + 1);
                oc[u] = ld_cg4(reinterpret_cast<const float4*>(R + d0));
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float f = expf(mc[u] - mt);
                lt = fmaf(lc[u], f, lt);
                acc.x = fmaf(oc[u].x, f, acc.x);
                acc.y = fmaf(oc[u].y, f, acc.y);
                acc.z = fmaf(oc[u].z, f, acc.z);
                acc.w = fmaf(oc[u].w, f, acc.w);
            }
        }
        for (; c < n_chunks; ++c) {
            const float* R = rec + (c * kNHead + h) * kRec;
            const float f = expf(ld_cg(R + kHeadDim) - mt);
            const float4 o = ld_cg4(reinterpret_cast<const float4*>(R + d0));
            lt = fmaf(ld_cg(R + kHeadDim + 1), f, lt);
            acc.x = fmaf(o.x, f, acc.x);
            acc.y = fmaf(o.y, f, acc.y);
            acc.z = fmaf(o.z, f, acc.z);
            acc.w = fmaf(o.w, f, acc.w);
        }
        const float inv = 1.0f / lt;
        stage_store(xs, bs, i, make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
    }
}

// One unit (8 Q4_0 blocks) of M rows against the staged input: w[m] is the
// unit's first byte in row m (16-byte aligned), xu the unit's 256 staged
// inputs, bu its 8 block sums, rot = unit index mod 8.  A 32-byte window
// (chunks k, k + 1) holds block k at window byte 2k.  Per block: low
// nibbles masked in place (0x0F), high nibbles masked in place (0xF0, so
// 16 n: their sum is scaled by 1/16), each byte moved into an otherwise
// zero word (the subnormal n 2^-149), products as packed f32x2 FMAs; the
// block sum less the precomputed offset term, scaled by d as the reference
// does per block (ops.cpp:495 matmul_q4_0).  The result carries 2^-49.
template <int M>
__device__ __forceinline__ void unit_dot_q4(const uint8_t* const (&w)[M], const float* xu, const float* bu, int rot,
                                            float (&out)[M]) {
    uint32_t win[M][8];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const uint4 c0 = *reinterpret_cast<const uint4*>(w[m]);
        win[m][0] = c0.x;
        win[m][1] = c0.y;
        win[m][2] = c0.z;
        win[m][3] = c0.w;
        out[m] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const uint4 c1 = *reinterpret_cast<const uint4*>(w[m] + 16 * (k + 1));
            win[m][4] = c1.x;
            win[m][5] = c1.y;
            win[m][6] = c1.z;
            win[m][7] = c1.w;
        }
        const int r0 = 2 * k;             // block k's first window byte
        const int w0 = (r0 + 2) >> 2;     // first window word holding its nibbles
        const float off = bu[k];
        float d[M];
        uint32_t lo[M][5], hi[M][5];
        uint64_t sl[M], sh[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const uint32_t dw = win[m][r0 >> 2];
            d[m] = h2f(static_cast<uint16_t>((r0 & 2) ? (dw >> 16) : (dw & 0xFFFFu)));
#pragma unroll
            for (int j = 0; j < 5; ++j) {
                const uint32_t v = (w0 + j < 8) ? win[m][w0 + j] : 0u;
                lo[m][j] = v & 0x0F0F0F0Fu;
                hi[m][j] = v & 0xF0F0F0F0u;
            }
            sl[m] = sh[m] = 0ull;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {   // inputs 4i..4i+3 of the block
            const float4 xv = *reinterpret_cast<const float4*>(xu + 32 * k + 4 * ((i + rot) & 7));
#pragma unroll
            for (int m = 0; m < M; ++m) {
#pragma unroll
                for (int e = 0; e < 4; e += 2) {
                    const int p0 = r0 + 2 + (i & 3) * 4 + e, p1 = p0 + 1;   // window bytes of the two weights
                    const uint32_t* src = (i < 4) ? lo[m] : hi[m];
                    const float a = __int_as_float(__byte_perm(src[(p0 >> 2) - w0], 0u, 0x4440u | (p0 & 3)));
                    const float b = __int_as_float(__byte_perm(src[(p1 >> 2) - w0], 0u, 0x4440u | (p1 & 3)));
                    const uint64_t xx = e == 0 ? pk2(xv.x, xv.y) : pk2(xv.z, xv.w);
                    if (i < 4) sl[m] = fma2(pk2(a, b), xx, sl[m]);
                    else sh[m] = fma2(pk2(a, b), xx, sh[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float2 a = up2(sl[m]), b = up2(sh[m]);
            out[m] = fmaf(d[m], fmaf(b.x + b.y, 0.0625f, a.x + a.y) - off, out[m]);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            win[m][0] = win[m][4];
            win[m][1] = win[m][5];
            win[m][2] = win[m][6];
            win[m][3] = win[m][7];
        }
    }
}

// Every (row, unit) pair of an nr-row product over `units` units, one per
// thread (nr * units <= PT): row r of matrix m at buf + (r + m * mstride) * stride.  Partials
// of matrix m go to part[m * PT + r * units + u] (the units of a row in adjacent threads).
template <int M>
__device__ __forceinline__ void rows_units(const uint8_t* buf, int stride, int mstride, int nr, int units,
                                           const float* xs, const float* bs, float* part) {
    const int p = threadIdx.x;   // nr * units <= PT (checked on the host)
    if (p < nr * units) {
        const int r = p / units, u = p - r * units;
        const uint8_t* w[M];
#pragma unroll
        for (int m = 0; m < M; ++m)
            w[m] = buf + static_cast<size_t>(r + m * mstride) * stride + u * kUnitBytes;
        float y[M];
        unit_dot_q4<M>(w, xs + u * kUnit, bs + 8 * u, u & 7, y);
#pragma unroll
        for (int m = 0; m < M; ++m) part[m * PT + p] = y[m];
    }
}

__device__ __forceinline__ float row_total(const float* part, int r, int nr, int units) {
    float y = 0.f;
    for (int u = 0; u < units; ++u) y += part[r * units + u];
    return y * kRowScale;
}

__global__ void __launch_bounds__(PT, 1) forward_persistent_kernel(const __grid_constant__ PersistArgs A) {
    extern __shared__ __align__(128) unsigned char psm[];
    float* xs = reinterpret_cast<float*>(psm);
    uint8_t* bufA = psm + A.off_a;
    uint8_t* bufB = psm + A.off_b;
    float* ks = reinterpret_cast<float*>(psm + A.off_kv);
    float* vs = ks + kAttRows * PKP;
    float* qs = vs + kAttRows * PKP;          // 8 heads x 64
    float* comb = qs + 8 * kHeadDim;          // 8 heads x kRec: the second half's (o, max, sum)
    float* part = reinterpret_cast<float*>(psm + A.off_part);   // 2 x PT
    __shared__ __align__(8) uint64_t wbar[2];
    __shared__ float red[PW];
    __shared__ float bsum[kPersistMaxBlocks];   // per 32-input block: 8 sum(x) 2^-49 of the staged input
    __shared__ int failed;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = static_cast<int>(gridDim.x), b = static_cast<int>(blockIdx.x);
    const int E = A.n_embd, KV = kNHeadKv * kHeadDim, FF = A.n_ff;
    const int rbE = E / 32 * 18, rbF = FF / 32 * 18;   // Q4_0 row bytes (n_embd, n_ff columns)
    const int uE = E / kUnit, uF = FF / kUnit;
    const int sE = A.stride_e, sF = A.stride_f;
    if (tid == 0) {
        mbar_init(&wbar[0], 1);
        mbar_init(&wbar[1], 1);
        fence_barrier_init();
        failed = 0;
    }
    __syncthreads();
    uint32_t useA = 0, useB = 0, nbar = 0;
    int r0q, r0e, r0f;
    const int nq = cta_rows(E + 2 * KV, b, G, r0q);
    const int ne = cta_rows(E, b, G, r0e);
    const int nf = cta_rows(FF, b, G, r0f);
    const int Rf = (FF + G - 1) / G;   // gate rows then up rows in buffer A, this many rows apart
    // attention chunk of this CTA (P2)
    const int L = A.pos + 1, C = A.att_chunks;
    const bool att = b < kNHeadKv * C;
    const int g = att ? b / C : 0, c = att ? b % C : 0;
    const int rr0 = c * kAttRows;
    const int nrows = att ? max(0, min(kAttRows, L - rr0)) : 0;
    const bool has_new = nrows > 0 && rr0 + nrows == L;
    const int ncached = has_new ? nrows - 1 : nrows;

    // lane 0 of warp 0: the CTA's rows of a product, one bulk copy per contiguous span
    auto span = [&](uint8_t* dst, const uint8_t* src, int bytes, uint64_t* bar) {
        if (bytes > 0) bulk_g2s_plain(dst, src, static_cast<uint32_t>(bytes), bar);
    };
    auto fill_qkv = [&](int l) {
        if (lane) return;
        const PersistLayer& Ly = A.layer[l];
        mbar_arrive_expect_tx(&wbar[0], static_cast<uint32_t>(nq * rbE));
        const int a0 = r0q, a1 = r0q + nq;            // rows of [q; k; v]
        const int q1 = min(a1, E), k0 = max(a0, E), k1 = min(a1, E + KV), v0 = max(a0, E + KV);
        span(bufA, Ly.w[0] + static_cast<size_t>(a0) * rbE, (q1 - a0) * rbE, &wbar[0]);
        span(bufA + static_cast<size_t>(k0 - a0) * rbE, Ly.w[1] + static_cast<size_t>(k0 - E) * rbE,
             (k1 - k0) * rbE, &wbar[0]);
        span(bufA + static_cast<size_t>(v0 - a0) * rbE, Ly.w[2] + static_cast<size_t>(v0 - E - KV) * rbE,
             (a1 - v0) * rbE, &wbar[0]);
    };
    auto fill_o = [&](int l) {
        if (lane) return;
        mbar_arrive_expect_tx(&wbar[1], static_cast<uint32_t>(ne * rbE));
        span(bufB, A.layer[l].w[3] + static_cast<size_t>(r0e) * rbE, ne * rbE, &wbar[1]);
    };
    auto fill_gu = [&](int l) {   // gate rows at 0, up rows Rf rows further
        if (lane) return;
        mbar_arrive_expect_tx(&wbar[0], static_cast<uint32_t>(2 * nf * rbE));
        span(bufA, A.layer[l].w[4] + static_cast<size_t>(r0f) * rbE, nf * rbE, &wbar[0]);
        span(bufA + static_cast<size_t>(Rf) * sE, A.layer[l].w[5] + static_cast<size_t>(r0f) * rbE, nf * rbE,
             &wbar[0]);
    };
    auto fill_down = [&](int l) {
        if (lane) return;
        mbar_arrive_expect_tx(&wbar[1], static_cast<uint32_t>(ne * rbF));
        span(bufB, A.layer[l].w[6] + static_cast<size_t>(r0e) * rbF, ne * rbF, &wbar[1]);
    };
    auto wait_buf = [&](int which) {
        uint32_t& u = which ? useB : useA;
        if (!failed && !mbar_wait(&wbar[which], u & 1)) {
            if (tid == 0) record_error(A.err, kErrWaitFull);
            // the copies may still land: wait once more before the buffer is reused or the CTA exits
            mbar_wait(&wbar[which], u & 1);
        }
        ++u;
    };
    auto barrier = [&]() {
        ++nbar;
        grid_barrier(A.sync, nbar * static_cast<uint32_t>(G), A.err, &failed);
    };
    auto block_sum = [&](float v) {   // every thread gets the CTA total (one barrier inside)
        v = warp_sum(v);
        if (lane == 0) red[warp] = v;
        __syncthreads();
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < PW; ++i) t += red[i];
        return t;
    };
    if (warp == 0) fill_qkv(0);

    for (int l = 0; l < A.n_layers; ++l) {
        const PersistLayer& Ly = A.layer[l];
        const size_t lbase = static_cast<size_t>(l) * A.n_ctx * KV;
        // ---- P1: rmsnorm + q/k/v (forward.cpp:184-196) ----
        if (warp == 0) fill_o(l);
        if (att) {   // this chunk's cached K/V rows of head g, for P2
            for (int e = tid; e < ncached * 32; e += PT) {
                const int r = e >> 5, piece = e & 31;
                const float* src = (piece < 16 ? A.key_cache : A.value_cache) + lbase +
                                   static_cast<size_t>(rr0 + r) * KV + g * kHeadDim + 4 * (piece & 15);
                float* dst = (piece < 16 ? ks : vs) + r * PKP + 4 * (piece & 15);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        const float ss1 = stage_rot(xs, bsum, A.x, Ly.attn_norm, E);
        const float rms1 = 1.0f / sqrtf(block_sum(ss1) / static_cast<float>(E) + A.eps);
        wait_buf(0);
        rows_units<1>(bufA, sE, 0, nq, uE, xs, bsum, part);
        __syncthreads();
        {
            // rope on the q and k rows here (ops.cpp:1223): a pair (2i, 2i + 1)
            // sits in adjacent threads (r0q is even); q also takes 1 / sqrt(64)
            float y = tid < nq ? row_total(part, tid, nq, uE) * rms1 : 0.f;
            const int r = r0q + tid;
            float partner = 0.f;
            if (warp < (nq + 31) / 32) partner = __shfl_xor_sync(0xffffffffu, y, 1);
            if (tid < nq) {
                if (r < E + KV) {
                    float sn, cs;
                    sincosf(static_cast<float>(A.pos) * A.inv_freq[(r & (kHeadDim - 1)) >> 1], &sn, &cs);
                    const float x0 = (r & 1) ? partner : y, x1 = (r & 1) ? y : partner;
                    y = (r & 1) ? x0 * sn + x1 * cs : x0 * cs - x1 * sn;
                }
                if (r < E) A.q[r] = y * 0.125f;
                else if (r < E + KV) A.k[r - E] = y;
                else A.v[r - E - KV] = y;
            }
        }
        barrier();
        // ---- P2: rope + attention + append (forward.cpp:198-208, ops.cpp:1223/1317) ----
        if (warp == 0) fill_gu(l);   // buffer A's reads ended before the barrier
        if (att) {
            asm volatile("cp.async.wait_all;" ::: "memory");
            if (warp < 8) {   // warp w: query head 8 g + w (rotated and scaled in P1)
                const int p = lane;
                const bool kv_row = has_new && warp < 2;   // warp 0 appends k, warp 1 v (rotated in P1)
                const float* qsrc = A.q + (8 * g + warp) * kHeadDim + 2 * p;
                const float* nsrc = (warp == 0 ? A.k : A.v) + g * kHeadDim + 2 * p;
                const float x0 = ld_cg(qsrc), x1 = ld_cg(qsrc + 1);
                const float n0 = kv_row ? ld_cg(nsrc) : 0.f, n1 = kv_row ? ld_cg(nsrc + 1) : 0.f;
                qs[warp * kHeadDim + 2 * p] = x0;
                qs[warp * kHeadDim + 2 * p + 1] = x1;
                if (kv_row) {   // keep, append (ops.cpp:1370-1371)
                    const size_t row = lbase + static_cast<size_t>(A.pos) * KV + g * kHeadDim;
                    float* sm = (warp == 0 ? ks : vs) + (nrows - 1) * PKP + 2 * p;
                    float* gl = (warp == 0 ? A.key_cache : A.value_cache) + row + 2 * p;
                    sm[0] = n0;
                    sm[1] = n1;
                    gl[0] = n0;
                    gl[1] = n1;
                }
            }
            __syncthreads();
            // warps 0-7: query heads 2 hp, 2 hp + 1 (hp = w & 3) over rows
            // [32 half, 32 half + 32) of the chunk (half = w >> 2); each K/V row
            // read from shared memory serves both heads
            if (warp < 8) {
                const int hp = warp & 3, half = warp >> 2;
                const float4* qa = reinterpret_cast<const float4*>(qs + (2 * hp) * kHeadDim);   // broadcast reads
                const float4* qb = reinterpret_cast<const float4*>(qs + (2 * hp + 1) * kHeadDim);
                const int r = 32 * half + lane;
                float sa = -INFINITY, sb = -INFINITY;
                if (r < nrows) {
                    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float4 kk = *reinterpret_cast<const float4*>(&ks[r * PKP + 4 * i]);
                        const float4 x = qa[i], y = qb[i];
                        a0 = fmaf(x.x, kk.x, a0);
                        a1 = fmaf(x.y, kk.y, a1);
                        a2 = fmaf(x.z, kk.z, a2);
                        a3 = fmaf(x.w, kk.w, a3);
                        b0 = fmaf(y.x, kk.x, b0);
                        b1 = fmaf(y.y, kk.y, b1);
                        b2 = fmaf(y.z, kk.z, b2);
                        b3 = fmaf(y.w, kk.w, b3);
                    }
                    sa = (a0 + a1) + (a2 + a3);
                    sb = (b0 + b1) + (b2 + b3);
                }
                float ma = sa, mb = sb;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, o));
                    mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
                }
                const float pa = (sa == -INFINITY) ? 0.f : expf(sa - ma);
                const float pb = (sb == -INFINITY) ? 0.f : expf(sb - mb);
                float la = pa, lb = pb;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    la += __shfl_xor_sync(0xffffffffu, la, o);
                    lb += __shfl_xor_sync(0xffffffffu, lb, o);
                }
                float oa0 = 0.f, oa1 = 0.f, ob0 = 0.f, ob1 = 0.f;
                const int nb = max(0, min(32, nrows - 32 * half));
                for (int j0 = 0; j0 < nb; j0 += 8) {   // eight rows' shuffles and loads in flight
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const int j = j0 + jj;   // < 32
                        const float wa = __shfl_sync(0xffffffffu, pa, j), wb = __shfl_sync(0xffffffffu, pb, j);
                        const float2 vv = *reinterpret_cast<const float2*>(&vs[(32 * half + j) * PKP + 2 * lane]);
                        if (j < nb) {
                            oa0 = fmaf(wa, vv.x, oa0);
                            oa1 = fmaf(wa, vv.y, oa1);
                            ob0 = fmaf(wb, vv.x, ob0);
                            ob1 = fmaf(wb, vv.y, ob1);
                        }
                    }
                }
                float* ca = comb + (2 * hp) * kRec;
                float* cb = comb + (2 * hp + 1) * kRec;
                if (half == 1) {
                    reinterpret_cast<float2*>(ca)[lane] = make_float2(oa0, oa1);
                    reinterpret_cast<float2*>(cb)[lane] = make_float2(ob0, ob1);
                    if (lane == 0) {
                        ca[kHeadDim] = ma;
                        ca[kHeadDim + 1] = la;
                        cb[kHeadDim] = mb;
                        cb[kHeadDim + 1] = lb;
                    }
                }
                __syncwarp();
                named_barrier_sync(1, 256);   // warps 0-7
                if (half == 0) {   // fold the second half (max -inf and sum 0 when it has no rows)
                    auto fold = [&](const float* cc, float m, float lsum, float o0, float o1, int hl) {
                        const float m1 = cc[kHeadDim], l1 = cc[kHeadDim + 1];
                        const float2 p1 = reinterpret_cast<const float2*>(cc)[lane];
                        const float mt = fmaxf(m, m1);
                        const float f0 = expf(m - mt), f1 = expf(m1 - mt);
                        float* R = A.partials + (static_cast<size_t>(c) * kNHead + 8 * g + hl) * kRec;
                        reinterpret_cast<float2*>(R)[lane] = make_float2(o0 * f0 + p1.x * f1, o1 * f0 + p1.y * f1);
                        if (lane == 0) {
                            R[kHeadDim] = mt;
                            R[kHeadDim + 1] = lsum * f0 + l1 * f1;
                        }
                    };
                    fold(ca, ma, la, oa0, oa1, 2 * hp);
                    fold(cb, mb, lb, ob0, ob1, 2 * hp + 1);
                }
            }
        }
        barrier();
        // ---- P3: x += Wo attn (forward.cpp:210-214) ----
        stage_attention(xs, bsum, A.partials, C, E);
        wait_buf(1);
        __syncthreads();
        rows_units<1>(bufB, sE, 0, ne, uE, xs, bsum, part);
        __syncthreads();
        if (tid < ne) A.x[r0e + tid] = ld_cg(A.x + r0e + tid) + row_total(part, tid, ne, uE);
        barrier();
        // ---- P4: rmsnorm + gate/up + SwiGLU (forward.cpp:216-227) ----
        if (warp == 0) fill_down(l);   // buffer B's reads ended before the barrier
        const float ss4 = stage_rot(xs, bsum, A.x, Ly.ffn_norm, E);
        const float rms4 = 1.0f / sqrtf(block_sum(ss4) / static_cast<float>(E) + A.eps);
        wait_buf(0);
        rows_units<2>(bufA, sE, Rf, nf, uE, xs, bsum, part);
        __syncthreads();
        if (tid < nf) {
            const float gg = row_total(part, tid, nf, uE) * rms4, uu = row_total(part + PT, tid, nf, uE) * rms4;
            // silu(g) * u (ops.cpp:1107-1113 then 1129-1146)
            A.hb[r0f + tid] = (gg * (1.0f / (1.0f + expf(-gg)))) * uu;
        }
        barrier();
        // ---- P5: x += Wdown hb (forward.cpp:227-229) ----
        if (warp == 0 && l + 1 < A.n_layers) fill_qkv(l + 1);   // buffer A's reads ended before the barrier
        stage_rot(xs, bsum, A.hb, nullptr, FF);
        wait_buf(1);
        __syncthreads();
        rows_units<1>(bufB, sF, 0, ne, uF, xs, bsum, part);
        __syncthreads();
        if (tid < ne) A.x[r0e + tid] = ld_cg(A.x + r0e + tid) + row_total(part, tid, ne, uF);
        if (l + 1 < A.n_layers) barrier();
    }
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       void** args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

template <int T, int EPI, bool TMA>
cudaError_t launch_gemv_k(const GemvArgs& a, int n_tiles, cudaStream_t stream) {
    static PerDeviceOnce once;
    const size_t smem = a.xs_bytes + (EPI == kEpiSwiGLU ? 2 : 1) * a.tile_bytes;
    cudaError_t e = once.run([&](int) {
        return cudaFuncSetAttribute(gemv_kernel<T, EPI, TMA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kGemvMaxSmem);
    });
    if (e != cudaSuccess) return e;
    GemvArgs copy = a;
    void* args[] = {&copy};
    return launch_pdl(reinterpret_cast<const void*>(gemv_kernel<T, EPI, TMA>), dim3(n_tiles), dim3(GT),
                      smem, stream, args);
}

template <int T, int EPI>
cudaError_t launch_gemv_t(const GemvArgs& a, int n_tiles, cudaStream_t stream) {
    return a.tile_bytes ? launch_gemv_k<T, EPI, true>(a, n_tiles, stream)
                        : launch_gemv_k<T, EPI, false>(a, n_tiles, stream);
}

template <int EPI>
cudaError_t launch_gemv_e(int type, const GemvArgs& a, int n_tiles, cudaStream_t stream) {
    switch (type) {
    case kWF32: return launch_gemv_t<kWF32, EPI>(a, n_tiles, stream);
    case kWF16: return launch_gemv_t<kWF16, EPI>(a, n_tiles, stream);
    case kWQ4_0: return launch_gemv_t<kWQ4_0, EPI>(a, n_tiles, stream);
    case kWQ8_0: return launch_gemv_t<kWQ8_0, EPI>(a, n_tiles, stream);
    case kWQ6_K: return launch_gemv_t<kWQ6_K, EPI>(a, n_tiles, stream);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace

int weight_row_bytes(int type, int cols) {
    switch (type) {
    case kWF32: return cols * 4;
    case kWF16: return cols * 2;
    case kWQ4_0: return cols % 32 ? -1 : cols / 32 * 18;
    case kWQ8_0: return cols % 32 ? -1 : cols / 32 * 34;
    case kWQ6_K: return cols % 256 ? -1 : cols / 256 * 210;
    default: return -1;
    }
}

size_t persist_smem_bytes(int n_embd, int n_ff, int grid, PersistArgs* a) {
    if (grid <= 0 || n_embd % kUnit || n_ff % kUnit || n_embd != kNHead * kHeadDim) return 0;
    auto stride = [](size_t rb) { return rb; };   // rows back to back (one bulk copy per span)
    const size_t rbE = n_embd / 32 * 18, rbF = n_ff / 32 * 18;
    const size_t sE = stride(rbE), sF = stride(rbF);
    const size_t Rq = (n_embd + 2 * kNHeadKv * kHeadDim + grid - 1) / grid;
    const size_t Re = (n_embd + grid - 1) / grid, Rf = (n_ff + grid - 1) / grid;
    // one (row, unit) pair per thread: every product's pairs fit one pass of the CTA
    const size_t uE = n_embd / kUnit, uF = n_ff / kUnit;
    if (std::max({Rq * uE, Rf * uE, Re * uE, Re * uF}) > static_cast<size_t>(PT)) return 0;
    if (Rq % 2) return 0;   // rope pairs must not straddle two CTAs
    if (std::max(n_embd, n_ff) / 32 > kPersistMaxBlocks) return 0;
    auto up128 = [](size_t v) { return (v + 127) / 128 * 128; };
    const size_t xs = up128(static_cast<size_t>(std::max(n_embd, n_ff)) * sizeof(float));
    const size_t bufA = up128(std::max(Rq, 2 * Rf) * sE);
    const size_t bufB = up128(std::max(Re * sE, Re * sF));
    const size_t kv = up128((2 * kAttRows * PKP + 8 * kHeadDim + 8 * kRec) * sizeof(float));
    const size_t part = 2 * PT * sizeof(float);
    const size_t total = xs + bufA + bufB + kv + part;
    if (total > 220 * 1024) return 0;
    a->stride_e = static_cast<int>(sE);
    a->stride_f = static_cast<int>(sF);
    a->off_a = static_cast<int>(xs);
    a->off_b = static_cast<int>(xs + bufA);
    a->off_kv = static_cast<int>(xs + bufA + bufB);
    a->off_part = static_cast<int>(xs + bufA + bufB + kv);
    return total;
}

int persist_max_chunks(int grid) { return grid / kNHeadKv; }

size_t persist_workspace_bytes(int grid) {
    return 256 + static_cast<size_t>(persist_max_chunks(grid)) * kNHead * kRec * sizeof(float);
}

cudaError_t launch_forward_persistent(const PersistArgs& a, int grid, size_t smem, cudaStream_t stream) {
    static PerDeviceOnce once;
    cudaError_t e = once.run([&](int) {
        return cudaFuncSetAttribute(forward_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    220 * 1024);
    });
    if (e != cudaSuccess) return e;
    // every CTA must be resident at once (the grid barriers): a cooperative launch
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(PT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, forward_persistent_kernel, a);
}

cudaError_t launch_gemv(int type, int epi, GemvArgs a, cudaStream_t stream) {
    const int n_mats = (epi == kEpiSwiGLU) ? 2 : 1;
    int rows = 0;
    bool tma = (a.row_bytes % 16) == 0;   // tiles of whole rows start 16-byte aligned
    for (int s = 0; s < a.n_seg; ++s) {
        rows += a.seg[s].rows;
        tma = tma && (reinterpret_cast<uintptr_t>(a.seg[s].W) & 15) == 0;
    }
    if (epi == kEpiSwiGLU) tma = tma && (reinterpret_cast<uintptr_t>(a.W2) & 15) == 0;
    if (rows == 0) return cudaSuccess;
    a.xs_bytes = (static_cast<int>(a.cols * sizeof(float)) + 15) & ~15;
    auto fits = [&](int rpc) {
        return a.xs_bytes + n_mats * static_cast<long>(rpc) * a.row_bytes <= kGemvMaxSmem;
    };
    a.ks = 1;
    a.rpc = GW * a.rpw;
    bool q4 = false;
    if (type == kWQ4_0 && tma) {
        // shared-memory Q4_0 path: groups of 4 rows, the columns split in
        // ks chunks so that short matrices still spread over many warps
        const int nb = a.cols >> 5;
        const int ks = rows >= 16384 ? 1 : (nb >= 128 ? 4 : (nb >= 48 ? 2 : 1));
        if (fits((GW / ks) * 4)) {
            a.ks = ks;
            a.rpc = (GW / ks) * 4;
            q4 = true;
        }
    }
    if (!q4) tma = tma && fits(a.rpc);
    a.tile_bytes = tma ? a.rpc * a.row_bytes : 0;
    int tiles = 0;
    for (int s = 0; s < a.n_seg; ++s) {
        a.seg[s].tile0 = tiles;
        tiles += (a.seg[s].rows + a.rpc - 1) / a.rpc;
    }
    if (uint32_t* w = nullptr; error_word(&w) == cudaSuccess) a.err = w;
    switch (epi) {
    case kEpiStore: return launch_gemv_e<kEpiStore>(type, a, tiles, stream);
    case kEpiAdd: return launch_gemv_e<kEpiAdd>(type, a, tiles, stream);
    case kEpiSwiGLU: return launch_gemv_e<kEpiSwiGLU>(type, a, tiles, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_embed(int type, float* x, const void* table, const int32_t* token, int n_vocab,
                         int n_embd, uint32_t* err, cudaStream_t stream) {
    const uint8_t* t = static_cast<const uint8_t*>(table);
    void* args[] = {&x, &t, &token, &n_vocab, &n_embd, &err};
    const int blocks = (n_embd + 255) / 256;
    if (type == kWF16)
        return launch_pdl(reinterpret_cast<const void*>(embed_kernel<kWF16>), dim3(blocks), dim3(256), 0,
                          stream, args);
    if (type == kWF32)
        return launch_pdl(reinterpret_cast<const void*>(embed_kernel<kWF32>), dim3(blocks), dim3(256), 0,
                          stream, args);
    return cudaErrorInvalidValue;
}

cudaError_t launch_argmax(const float* logits, int n, int32_t* out, cudaStream_t stream) {
    void* args[] = {&logits, &n, &out};
    return launch_pdl(reinterpret_cast<const void*>(argmax_kernel), dim3(1), dim3(1024), 0, stream, args);
}

cudaError_t launch_sample(float* logits, int n, float temperature, float top_p, float r, bool use_top_p,
                          int32_t* out, cudaStream_t stream) {
    static PerDeviceOnce once;
    cudaError_t e = once.run([&](int) {
        cudaError_t x = cudaFuncSetAttribute(sample_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSampleMaxSmem);
        if (x != cudaSuccess) return x;
        return cudaFuncSetAttribute(sample_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kSampleMaxSmem);
    });
    if (e != cudaSuccess) return e;
    const size_t smem = (static_cast<size_t>((n + 3) & ~3) + (use_top_p ? 2 * kTopPMax : 0)) * 4;
    void* args[] = {&logits, &n, &temperature, &top_p, &r, &out};
    return launch_pdl(use_top_p ? reinterpret_cast<const void*>(sample_kernel<true>)
                                : reinterpret_cast<const void*>(sample_kernel<false>),
                      dim3(1), dim3(kSampleThreads), smem, stream, args);
}

cudaError_t launch_rmsnorm(float* out, const float* x, const float* w, int n, float eps,
                           cudaStream_t stream) {
    void* args[] = {&out, &x, &w, &n, &eps};
    return launch_pdl(reinterpret_cast<const void*>(rmsnorm_kernel), dim3(1), dim3(1024), 0, stream, args);
}

cudaError_t launch_vec_add(float* out, const float* x, int n, cudaStream_t stream) {
    void* args[] = {&out, &x, &n};
    const int blocks = min((n + 255) / 256, 1024);
    return launch_pdl(reinterpret_cast<const void*>(vec_add_kernel), dim3(blocks), dim3(256), 0, stream,
                      args);
}

}  // namespace tle
