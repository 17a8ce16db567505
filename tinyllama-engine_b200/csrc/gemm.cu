// gemm.cu -- the batched prompt: every product of forward() for S prompt
// tokens at once, on the tcgen05 tensor cores.
//
// Reference semantics: generate.cpp:52-59 feeds the prompt one token at a
// time through forward() (forward.cpp:178-265), so each weight matrix meets
// one vector per call (matmul, ops.cpp:959-981).  For S prompt tokens the
// products of one layer are the matrix products Y[S][rows] = X[S][cols] W^T
// of the same weights with S inputs.
//
// B200 design:
//  * The weights are dequantised once into an fp16 copy (launch_pack_f16:
//    the reference's dequantised value of every GGUF format, rounded to
//    fp16; 2 bytes a weight, ~1.9 GB for TinyLlama-1.1B, kept resident in
//    HBM next to the GGUF bytes the decode path reads).
//  * gemm_f16_kernel: one CTA per (128 weight rows, 128 tokens) tile.  A
//    producer warp streams 64-wide K slices of the weight tile (TMA, 128-byte
//    swizzle) and of the token tile into a ring of shared-memory stages; one
//    thread of the MMA warp issues tcgen05.mma kind::f16 (M = 128 weight
//    rows = TMEM lanes, N = 128 tokens = TMEM columns, fp32 accumulation in
//    TMEM); the four warps read the accumulator back (one weight row per
//    thread) and apply the epilogue the token-at-a-time path fuses into its
//    GEMV: store into q/k/v, residual add, or SwiGLU of a gate and an up
//    accumulator (two per CTA) written as fp16 for the down product.
//  * Small kernels around it: the embedding rows, RMSNorm of S rows into the
//    fp16 operand, and the fp16 copy of the attention output.
// Operands enter the tensor cores as fp16 (11-bit significand) with fp32
// accumulation; the attention in between is tle_prefill's (bf16 operands).
#include <cuda.h>
#include <cuda_fp16.h>
#include <math.h>
#include <stddef.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace cg = cooperative_groups;

namespace tle {

namespace {

constexpr int GM = kGemmTileRows;     // 128 weight rows: TMEM lanes
constexpr int GN = kGemmTileTokens;   // 128 tokens: TMEM columns per accumulator
constexpr int GK = kGemmTileK;        // 64 fp16 = one 128-byte swizzle row
constexpr int kGemmThreads = 256;
constexpr uint32_t kTileBytes = GM * GK * 2;   // 16 KB, the same for a token tile
static_assert(GM == GN, "weight and token tiles share one tensor-map box");
constexpr uint32_t kIdesc = idesc_f16_f32(GM, GN);

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
// f2h for activations: a finite value whose fp16 rounding overflows (|f| >=
// 65520) is reported (0x109) instead of silently entering the next product
// as inf.
__device__ __forceinline__ uint16_t f2h_checked(float f, uint32_t* err) {
    const uint16_t h = f2h(f);
    if ((h & 0x7FFFu) == 0x7C00u && fabsf(f) < INFINITY) record_error(err, kErrF16Range);
    return h;
}

// Bounded wait; after the first expiry in a thread every later wait of that
// thread returns at once.
__device__ __forceinline__ void wait_or_flag(uint64_t* bar, uint32_t parity, uint32_t* err,
                                             uint32_t code, bool& failed) {
    if (failed) return;
    if (!mbar_wait(bar, parity)) {
        record_error(err, code);
        failed = true;
    }
}

template <int NACC, int STAGES>
struct GemmSmem {
    uint16_t a[STAGES][NACC][GM * GK];   // weight slices (gate, up), SW128 K-major
    uint16_t b[STAGES][GN * GK];         // token slices
    uint64_t full[STAGES];               // the stage's copies landed
    uint64_t empty[STAGES];              // the stage's MMAs completed
    uint64_t acc_full;                   // the last MMA completed
    uint64_t drain;                      // failure path: every MMA issued so far completed
    int issued, consumed;                // failure path: K blocks copied / taken by the MMAs
    uint32_t tmem_base;
};
template <int EPI>
struct GemmCfg {
    static constexpr int NACC = EPI == kEpiSwiGLU ? 2 : 1;
    static constexpr int STAGES = NACC == 2 ? 4 : 6;
    static constexpr uint32_t kCols = NACC * GN;   // TMEM columns (128 or 256)
    using Smem = GemmSmem<NACC, STAGES>;
    static constexpr int kSmemBytes = static_cast<int>(sizeof(Smem)) + 1024;   // + alignment slack
};

struct GemmArgs {
    CUtensorMap tm_w;   // fp16 [w_rows][K], box {64, 128}
    CUtensorMap tm_x;   // fp16 [S_pad][K], box {64, 128}
    int K;
    int n_tokens;
    int up_row0;        // SwiGLU: first up row in tm_w (= n_ff)
    int n_seg;
    int seg_row0[3];
    int seg_rows[3];
    float* seg_out[3];
    uint16_t* h_out;    // SwiGLU: [S_pad][up_row0]
    uint32_t* err;
};

// Warp roles (256 threads, one CTA per SM by shared memory):
//   warp 0: TMA producer (one lane issues), warp 1: MMA issuer (one elected
//   lane); then all eight warps run the epilogue, warp w on TMEM lanes
//   32 (w % 4) .. +31 (the lanes a warp may access are fixed by its rank mod
//   4) and token half w / 4 of the tile.
template <int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_f16_kernel(const __grid_constant__ GemmArgs A) {
    using C = GemmCfg<EPI>;
    constexpr int NACC = C::NACC;
    constexpr int ST = C::STAGES;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // SW128 atoms need 1024-byte aligned tiles (the launch adds 1 KB of slack)
    typename C::Smem& S = *reinterpret_cast<typename C::Smem*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * GM;
    const int t0 = blockIdx.y * GN;
    // split z of n_split: K blocks [kb0, kb1)
    const int n_split = static_cast<int>(gridDim.z), z = static_cast<int>(blockIdx.z);
    const int nk_all = A.K / GK;
    const int kb0 = z * nk_all / n_split;
    const int nk = (z + 1) * nk_all / n_split - kb0;

    // Programmatic dependent launch: the next kernel on the stream may be
    // scheduled now; it waits for this grid before touching its outputs.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        mbar_init(&S.acc_full, 1);
        mbar_init(&S.drain, 1);
        S.issued = 0;
        S.consumed = 0;
        fence_barrier_init();
        prefetch_tmap(&A.tm_w);
        prefetch_tmap(&A.tm_x);
    }
    if (warp == 0) {
        tmem_alloc(&S.tmem_base, C::kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    bool failed = false;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        // No kernel writes the weights, so the first stages' weight slices
        // stream while the previous kernel on the stream (the producer of the
        // token operand) finishes; the token slices, and everything else
        // this grid reads or writes, wait for it (griddepcontrol.wait).
        const int pre = nk < ST ? nk : ST;
        if (lane == 0) {
            for (int kb = 0; kb < pre; ++kb) {
                const int kx = (kb0 + kb) * GK;
                mbar_arrive_expect_tx(&S.full[kb], (NACC + 1) * kTileBytes);
                tma_load_2d(S.a[kb][0], &A.tm_w, kx, m0, &S.full[kb]);
                if (NACC == 2) tma_load_2d(S.a[kb][NACC - 1], &A.tm_w, kx, A.up_row0 + m0, &S.full[kb]);
            }
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane == 0) {
            for (int kb = 0; kb < pre; ++kb) tma_load_2d(S.b[kb], &A.tm_x, (kb0 + kb) * GK, t0, &S.full[kb]);
            S.issued = pre;
        }
        __syncwarp();
        for (int kb = pre; kb < nk; ++kb) {
            const int s = kb % ST;
            wait_or_flag(&S.empty[s], ((kb / ST) - 1) & 1, A.err, kErrWaitEmpty, failed);
            failed = __any_sync(0xffffffffu, failed);   // the warp stops as one
            if (failed) break;
            if (lane == 0) {
                const int kx = (kb0 + kb) * GK;
                mbar_arrive_expect_tx(&S.full[s], (NACC + 1) * kTileBytes);
                tma_load_2d(S.a[s][0], &A.tm_w, kx, m0, &S.full[s]);
                if (NACC == 2) tma_load_2d(S.a[s][NACC - 1], &A.tm_w, kx, A.up_row0 + m0, &S.full[s]);
                tma_load_2d(S.b[s], &A.tm_x, kx, t0, &S.full[s]);
                S.issued = kb + 1;
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        // ------------------------------ MMA issuer --------------------------------
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % ST;
            wait_or_flag(&S.full[s], (kb / ST) & 1, A.err, kErrWaitFull, failed);
            failed = __any_sync(0xffffffffu, failed);
            if (failed) break;
            if (lane == 0) S.consumed = kb + 1;
            tc_fence_after();
            if (elect_one()) {
                const uint64_t db = sw128_desc(smem_u32(S.b[s]));
#pragma unroll
                for (int acc = 0; acc < NACC; ++acc) {
                    const uint64_t da = sw128_desc(smem_u32(S.a[s][acc]));
#pragma unroll
                    for (int kk = 0; kk < GK / 16; ++kk)   // 16 fp16 = 32 bytes = 2 descriptor units
                        umma_bf16(tmem + acc * GN, da + 2 * kk, db + 2 * kk, kIdesc,
                                  (kb > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&S.empty[s]);
                if (kb == nk - 1) umma_commit(&S.acc_full);
            }
            __syncwarp();
        }
    }

    // ------------------------------ epilogue (all warps) ------------------------------
    if (warp >= 2) asm volatile("griddepcontrol.wait;" ::: "memory");   // the epilogue reads / writes outputs
    wait_or_flag(&S.acc_full, 0, A.err, kErrWaitMma, failed);
    tc_fence_after();
    const int quad = warp & 3, half = warp >> 2;
    const int row_in_tile = 32 * quad + lane;
    const int r = m0 + row_in_tile;   // this thread's weight row
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * quad) << 16);
    float* seg_out = nullptr;
    int seg_ld = 0;
    if (EPI != kEpiSwiGLU) {
        // a tile lies inside one segment (the launcher checks it)
        int si = 0;
        for (int i = 1; i < A.n_seg; ++i)
            if (m0 >= A.seg_row0[i]) si = i;
        seg_ld = A.seg_rows[si];
        seg_out = A.seg_out[si] + (r - A.seg_row0[si]);
    }
    // The epilogue of tokens [tb, te) of this thread's row from v (and u):
    // store, residual add (all loads of the chunk before its stores, so
    // they overlap), or SwiGLU (ops.cpp:1107-1113 then 1129-1146).
    auto finish = [&](int tb, int n, const float (&v)[32], const float (&u)[32]) {
        if (EPI == kEpiStore) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < n && tb + j < A.n_tokens) seg_out[static_cast<size_t>(tb + j) * seg_ld] = v[j];
        } else if (EPI == kEpiAdd) {
            float x[32];
#pragma unroll
            for (int j = 0; j < 32; ++j)
                x[j] = (j < n && tb + j < A.n_tokens) ? seg_out[static_cast<size_t>(tb + j) * seg_ld] : 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < n && tb + j < A.n_tokens) seg_out[static_cast<size_t>(tb + j) * seg_ld] = x[j] + v[j];
        } else {
            // silu(g) u with the fast exponential and division: the result
            // is rounded to fp16 (11 bits), far coarser than their error
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                if (j < n && tb + j < A.n_tokens) {
                    const float g = v[j];
                    A.h_out[static_cast<size_t>(tb + j) * A.up_row0 + r] =
                        f2h_checked(__fdividef(g, 1.0f + __expf(-g)) * u[j], A.err);
                }
            }
        }
    };
    if (n_split == 1) {
#pragma unroll 1
        for (int c = 2 * half; c < 2 * half + 2; ++c) {
            float v[32];
            float u[32];
            tmem_ld32(trow + 32 * c, v);
            if (NACC == 2) tmem_ld32(trow + GN + 32 * c, u);
            tmem_wait_ld();
            finish(t0 + 32 * c, 32, v, u);
        }
    } else {
        // Split K over the CTAs of a cluster (one per split).  Split z owns
        // tokens [z per, (z+1) per) of the output.  Once every split's MMAs
        // have completed (first cluster barrier: the stage memory of every
        // CTA is idle), each split pushes its fp32 accumulators, token slice
        // by token slice, into the owning CTA's shared memory with remote
        // stores (slot (acc, split) of a row padded to per + 4 floats, so
        // 16-byte accesses hit distinct bank groups); after the second
        // barrier each CTA adds up its slots in split order (deterministic)
        // from its own memory and runs the epilogue.  Remote stores expose no
        // round trip, where remote loads cost one per slice and split.
        float* red = reinterpret_cast<float*>(&S.a[0][0][0]);
        static_assert(offsetof(typename C::Smem, b) == sizeof(S.a) &&
                          sizeof(S.a) + sizeof(S.b) >= sizeof(float) * NACC * GM * (GN + 4 * 8),
                      "the slots of up to 8 splits fit the stage ring");
        const int per = GN / n_split;   // 16, 32, 64 or 128 tokens
        const int rps = per + 4;
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();
#pragma unroll 1
        for (int acc = 0; acc < NACC; ++acc) {
#pragma unroll 1
            for (int c = 2 * half; c < 2 * half + 2; ++c) {
                float v[32];
                tmem_ld32(trow + acc * GN + 32 * c, v);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int tk = 32 * c + 4 * j;   // a 4-token group never straddles two owners
                    const int dst = tk / per;
                    float* peer = cl.map_shared_rank(red, dst);
                    *reinterpret_cast<float4*>(peer + ((acc * n_split + z) * GM + row_in_tile) * rps + (tk - dst * per)) =
                        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                }
            }
        }
        cl.sync();
        const int hb = per / 2;   // this warp's half of the CTA's tokens
        for (int tb = half * hb; tb < (half + 1) * hb; tb += 32) {
            const int n = (half + 1) * hb - tb < 32 ? (half + 1) * hb - tb : 32;
            float v[32];
            float u[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = u[j] = 0.f;
            for (int zz = 0; zz < n_split; ++zz) {
                const float* sa = red + (zz * GM + row_in_tile) * rps + tb;
                const float* sb = red + ((n_split + zz) * GM + row_in_tile) * rps + tb;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (4 * q < n) {
                        const float4 a4 = *reinterpret_cast<const float4*>(sa + 4 * q);
                        v[4 * q] += a4.x; v[4 * q + 1] += a4.y; v[4 * q + 2] += a4.z; v[4 * q + 3] += a4.w;
                        if (NACC == 2) {
                            const float4 b4 = *reinterpret_cast<const float4*>(sb + 4 * q);
                            u[4 * q] += b4.x; u[4 * q + 1] += b4.y; u[4 * q + 2] += b4.z; u[4 * q + 3] += b4.w;
                        }
                    }
                }
            }
            finish(t0 + z * per + tb, n, v, u);
        }
    }
    // Failure path (a bounded wait expired somewhere in the CTA): nothing the
    // CTA issued may still write shared or tensor memory when the memory is
    // freed, so wait (bounded) for the copies no MMA took and for a final
    // commit of the MMA thread's work; a drain that expires is reported too.
    tc_fence_before();
    if (__syncthreads_or(failed ? 1 : 0)) {
        bool drained = true;
        if (warp == 1 && elect_one()) {
            umma_commit(&S.drain);
            drained = mbar_wait(&S.drain, 0);
        }
        if (threadIdx.x == 0)
            for (int kb = S.consumed; kb < S.issued; ++kb)
                if (!mbar_wait(&S.full[kb % ST], (kb / ST) & 1)) {
                    drained = false;
                    break;
                }
        if (!drained) record_error(A.err, kErrDrain);
        __syncthreads();
    }
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kCols);
    }
}

// ---- fp16 copy of a GGUF weight ---------------------------------------------
// Element e of a row, dequantised as the reference does (gguf block layouts,
// ops.cpp Q4_0 616-655, Q8_0 442-473, Q6_K 882-948): the products are exact
// in fp32, so the only rounding is the final one to fp16.
template <int T>
__device__ __forceinline__ float deq(const uint8_t* row, int e);
template <>
__device__ __forceinline__ float deq<kWF32>(const uint8_t* row, int e) {
    return reinterpret_cast<const float*>(row)[e];
}
template <>
__device__ __forceinline__ float deq<kWF16>(const uint8_t* row, int e) {
    return h2f(reinterpret_cast<const uint16_t*>(row)[e]);
}
template <>
__device__ __forceinline__ float deq<kWQ4_0>(const uint8_t* row, int e) {
    const uint8_t* blk = row + 18 * (e >> 5);
    const int j = e & 31;
    const float d = h2f(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
    const int q = blk[2 + (j & 15)];
    const int n = (j < 16) ? (q & 15) : (q >> 4);
    return static_cast<float>(n - 8) * d;
}
template <>
__device__ __forceinline__ float deq<kWQ8_0>(const uint8_t* row, int e) {
    const uint8_t* blk = row + 34 * (e >> 5);
    const float d = h2f(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
    return static_cast<float>(static_cast<int8_t>(blk[2 + (e & 31)])) * d;
}
template <>
__device__ __forceinline__ float deq<kWQ6_K>(const uint8_t* row, int e) {
    // super-block of 256: half h, quarter i of the half, position l
    const uint8_t* blk = row + 210 * (e >> 8);
    const int r = e & 255;
    const int h = r >> 7, i = (r >> 5) & 3, l = r & 31;
    const uint32_t ql = blk[64 * h + l + 32 * (i & 1)];
    const uint32_t qh = blk[128 + 32 * h + l];
    const int q = static_cast<int>(((i < 2) ? (ql & 15u) : (ql >> 4)) | (((qh >> (2 * i)) & 3u) << 4)) - 32;
    const float d = h2f(static_cast<uint16_t>(blk[208] | (blk[209] << 8)));
    const int8_t sc = static_cast<int8_t>(blk[192 + 8 * h + (l >> 4) + 2 * i]);
    return d * static_cast<float>(sc) * static_cast<float>(q);
}

template <int T>
__global__ void __launch_bounds__(256) pack_f16_kernel(uint16_t* __restrict__ dst, const uint8_t* __restrict__ W,
                                                       int rows, int cols, int row_bytes) {
    const size_t n = static_cast<size_t>(rows) * cols;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t rr = i / static_cast<size_t>(cols);
        const int e = static_cast<int>(i - rr * static_cast<size_t>(cols));
        dst[i] = f2h(deq<T>(W + rr * static_cast<size_t>(row_bytes), e));
    }
}

// ---- RMSNorm of S rows into the fp16 operand (ops.cpp:1040-1054 per row) ----
// The row kernels below run as programmatic dependents: they trigger the
// next launch and wait for the previous kernel before their first load.  Data
// the previous kernel wrote is read through plain pointers, which the
// compiler may not hoist above the wait.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__global__ void __launch_bounds__(256) rmsnorm_rows_f16_kernel(uint16_t* out, const float* x, const float* w, int n,
                                                               float eps, uint32_t* err) {
    __shared__ float red[8];
    __shared__ float rms;
    pdl_enter();
    const float* xr = x + static_cast<size_t>(blockIdx.x) * n;
    uint16_t* orow = out + static_cast<size_t>(blockIdx.x) * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += 256) ss = fmaf(xr[i], xr[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < 8; ++i) t += red[i];
        rms = 1.0f / sqrtf(t / static_cast<float>(n) + eps);
    }
    __syncthreads();
    const float s = rms;
    for (int i = threadIdx.x; i < n; i += 256) orow[i] = f2h_checked(xr[i] * s * w[i], err);
}

__global__ void __launch_bounds__(256) to_f16_kernel(uint16_t* out, const float* x, size_t n, uint32_t* err) {
    pdl_enter();
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = f2h_checked(x[i], err);
}

// embed_token (forward.cpp:35-60) for S tokens: block (x, t) writes a slice
// of row t.  A token outside [0, n_vocab) is reported (0x106) and gives zeros.
template <int T>
__global__ void __launch_bounds__(256) embed_rows_kernel(float* x, const uint8_t* table, const int32_t* tokens,
                                                         int n_vocab, int n_embd, uint32_t* err) {
    pdl_enter();
    const int t = blockIdx.y;
    const int tok = tokens[t];
    const bool ok = tok >= 0 && tok < n_vocab;
    if (!ok && threadIdx.x == 0 && blockIdx.x == 0) record_error(err, kErrBadToken);
    float* xr = x + static_cast<size_t>(t) * n_embd;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_embd; i += gridDim.x * blockDim.x) {
        float v = 0.f;
        if (ok) {
            const size_t e = static_cast<size_t>(tok) * n_embd + i;
            v = (T == kWF16) ? h2f(reinterpret_cast<const uint16_t*>(table)[e])
                             : reinterpret_cast<const float*>(table)[e];
        }
        xr[i] = v;
    }
}

template <int EPI>
cudaError_t launch_gemm_e(const GemmArgs& a, dim3 grid, cudaStream_t stream) {
    using C = GemmCfg<EPI>;
    static PerDeviceOnce once;
    cudaError_t e = once.run([&](int) {
        cudaError_t r = cudaFuncSetAttribute(gemm_f16_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::kSmemBytes);
        if (r != cudaSuccess) return r;
        return cudaFuncSetAttribute(gemm_f16_kernel<EPI>, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    });
    if (e != cudaSuccess) return e;
    // the K splits of a tile form one cluster (z): they are co-scheduled and
    // reduce through distributed shared memory
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(C::kSmemBytes);
    cfg.stream = stream;
    // and a programmatic dependent of the previous kernel on the stream
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = grid.z;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, gemm_f16_kernel<EPI>, a);
}

inline int grid_for(size_t n) {
    const size_t b = (n + 255) / 256;
    return static_cast<int>(b < 148 * 16 ? (b ? b : 1) : 148 * 16);
}

// A row kernel of the prompt pass as a programmatic dependent of the
// previous kernel on the stream (the kernels wait with griddepcontrol.wait
// before their first load).
template <typename... P, typename... Arg>
cudaError_t launch_row_kernel(void (*fn)(P...), dim3 grid, cudaStream_t stream, Arg... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, static_cast<P>(args)...);
}

}  // namespace

cudaError_t launch_gemm_f16(int epi, const GemmLaunch& g, cudaStream_t stream) {
    if (g.K <= 0 || g.K % GK || g.tile_rows <= 0 || g.tile_rows % GM || g.n_tokens <= 0)
        return cudaErrorInvalidValue;
    if (epi == kEpiSwiGLU ? (g.w_rows != 2 * g.tile_rows || !g.h_out) : (g.w_rows != g.tile_rows))
        return cudaErrorInvalidValue;
    GemmArgs a{};
    const int s_pad = (g.n_tokens + GN - 1) / GN * GN;
    cudaError_t e = make_tmap_16b(&a.tm_w, const_cast<uint16_t*>(g.W), static_cast<uint64_t>(g.K),
                                  static_cast<uint64_t>(g.w_rows), GM, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    if (e != cudaSuccess) return e;
    e = make_tmap_16b(&a.tm_x, const_cast<uint16_t*>(g.X), static_cast<uint64_t>(g.K),
                      static_cast<uint64_t>(s_pad), GN, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    if (e != cudaSuccess) return e;
    a.K = g.K;
    a.n_tokens = g.n_tokens;
    a.up_row0 = g.tile_rows;
    a.h_out = g.h_out;
    a.err = g.err;
    const int n_split = g.n_split > 1 ? g.n_split : 1;
    if (n_split > 8 || (n_split & (n_split - 1)) || n_split > g.K / GK) return cudaErrorInvalidValue;
    if (epi != kEpiSwiGLU) {
        // segments: in row order, tile-aligned, covering [0, w_rows)
        if (g.n_seg < 1 || g.n_seg > 3) return cudaErrorInvalidValue;
        int next = 0;
        for (int i = 0; i < g.n_seg; ++i) {
            if (g.seg[i].row0 != next || g.seg[i].rows <= 0 || g.seg[i].rows % GM || !g.seg[i].out)
                return cudaErrorInvalidValue;
            next += g.seg[i].rows;
            a.seg_row0[i] = g.seg[i].row0;
            a.seg_rows[i] = g.seg[i].rows;
            a.seg_out[i] = g.seg[i].out;
        }
        if (next != g.w_rows) return cudaErrorInvalidValue;
        a.n_seg = g.n_seg;
    }
    const dim3 grid(g.tile_rows / GM, s_pad / GN, n_split);
    switch (epi) {
        case kEpiStore: return launch_gemm_e<kEpiStore>(a, grid, stream);
        case kEpiAdd: return launch_gemm_e<kEpiAdd>(a, grid, stream);
        case kEpiSwiGLU: return launch_gemm_e<kEpiSwiGLU>(a, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_pack_f16(int type, uint16_t* dst, const void* W, int rows, int cols, cudaStream_t stream) {
    const int rb = weight_row_bytes(type, cols);
    if (rb <= 0 || rows <= 0) return cudaErrorInvalidValue;
    const int grid = grid_for(static_cast<size_t>(rows) * cols);
    const uint8_t* w = static_cast<const uint8_t*>(W);
    switch (type) {
        case kWF32: pack_f16_kernel<kWF32><<<grid, 256, 0, stream>>>(dst, w, rows, cols, rb); break;
        case kWF16: pack_f16_kernel<kWF16><<<grid, 256, 0, stream>>>(dst, w, rows, cols, rb); break;
        case kWQ4_0: pack_f16_kernel<kWQ4_0><<<grid, 256, 0, stream>>>(dst, w, rows, cols, rb); break;
        case kWQ8_0: pack_f16_kernel<kWQ8_0><<<grid, 256, 0, stream>>>(dst, w, rows, cols, rb); break;
        case kWQ6_K: pack_f16_kernel<kWQ6_K><<<grid, 256, 0, stream>>>(dst, w, rows, cols, rb); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows_f16(uint16_t* out, const float* x, const float* w, int n, float eps,
                                    int n_tokens, uint32_t* err, cudaStream_t stream) {
    if (n <= 0 || n_tokens <= 0) return cudaErrorInvalidValue;
    return launch_row_kernel(rmsnorm_rows_f16_kernel, dim3(n_tokens), stream, out, x, w, n, eps, err);
}

cudaError_t launch_to_f16(uint16_t* out, const float* x, size_t n, uint32_t* err, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    return launch_row_kernel(to_f16_kernel, dim3(grid_for(n)), stream, out, x, n, err);
}

cudaError_t launch_embed_rows(int type, float* x, const void* table, const int32_t* tokens, int n_tokens,
                              int n_vocab, int n_embd, uint32_t* err, cudaStream_t stream) {
    if (n_tokens <= 0 || n_embd <= 0 || n_tokens > 65535) return cudaErrorInvalidValue;
    const dim3 grid((n_embd + 255) / 256, n_tokens);
    const uint8_t* tb = static_cast<const uint8_t*>(table);
    if (type == kWF16) return launch_row_kernel(embed_rows_kernel<kWF16>, grid, stream, x, tb, tokens, n_vocab, n_embd, err);
    if (type == kWF32) return launch_row_kernel(embed_rows_kernel<kWF32>, grid, stream, x, tb, tokens, n_vocab, n_embd, err);
    return cudaErrorInvalidValue;
}

}  // namespace tle
