// prefill.cu -- causal prefill attention on the tcgen05 tensor cores.
//
// Reference semantics: the reference prefills one token at a time
// (generate.cpp:56-59), i.e. for i = 0..S-1 rope(q_i, k_i, pos0+i)
// (ops.cpp:1223) then attention(..., pos0+i) (ops.cpp:1317): token i appends
// its rotated k and v at row pos0+i and attends to cache rows 0..pos0+i.
// That is causal attention over the cache prefix plus the S new rows.
//
// B200 design, two launches:
//  1. prefill_prep_kernel (HBM-bound): rotates q and k in fp32 (the rotation
//     the reference applies), appends rotated k and v to the fp32 cache, and
//     writes bf16 operands for the tensor cores into the workspace:
//        Qb [32 heads][S_pad][64]   rotated q * 1/8 (exact power-of-two scale)
//        Kb [4 kv][R_pad][64]       rotated k (rows < pos0 from the cache)
//        Vt [4 kv][64][R_pad]       v transposed so PV's B operand is K-major
//     (R = pos0 + S rows; pads are zero).
//  2. prefill_attn_kernel: one CTA per (128-query tile, query head).  TMA
//     (SWIZZLE_128B, no multicast) loads the Q tile once and double-buffers
//     128-row K / V^T tiles of the head's KV head; one thread issues
//     S = Q K^T (M=128, N=128, K=64) into TMEM; 128 threads (one per query
//     row) read S back, apply the causal mask and an fp32 online softmax,
//     write P (bf16) into shared memory in the swizzled K-major layout; the
//     same thread issues O_j = P V_j (M=128, N=64, K=128) into TMEM; the rows
//     accumulate O in registers with the softmax rescale.  Q, K, V and P
//     enter the MMA as bf16 with fp32 accumulation (the north-star prefill
//     contract, tolerance 2e-2).
#include <cuda.h>
#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace tle {

namespace {

constexpr int HD = kHeadDim;   // 64
constexpr int NH = kNHead;     // 32
constexpr int NKV = kNHeadKv;  // 4
constexpr int GQA = NH / NKV;  // 8
constexpr int BM = 128;        // query rows per CTA
constexpr int BN = 128;        // kv rows per tile
constexpr int ATTN_THREADS = 128;
constexpr uint32_t TMEM_COLS = 256;  // S: cols [0,128), O_j: cols [128,192)
constexpr float kQScale = 0.125f;    // 1/sqrt(64)
constexpr float kLog2e = 1.4426950408889634f;

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

struct Layout {
    int S_pad, R, R_pad;
    size_t qb_off, kb_off, vt_off, total;
};

inline Layout layout_for(int n_tokens, int pos0) {
    Layout L;
    L.S_pad = round_up(n_tokens, BM);
    L.R = pos0 + n_tokens;
    L.R_pad = round_up(L.R, BN);
    L.qb_off = 0;
    L.kb_off = L.qb_off + static_cast<size_t>(NH) * L.S_pad * HD * 2;
    L.vt_off = L.kb_off + static_cast<size_t>(NKV) * L.R_pad * HD * 2;
    L.total = L.vt_off + static_cast<size_t>(NKV) * HD * L.R_pad * 2;
    return L;
}

struct PrepArgs {
    const float* q;
    const float* k;
    const float* v;
    float* kc;  // layer base of the key cache: [n_ctx][256]
    float* vc;
    __nv_bfloat16* qb;
    __nv_bfloat16* kb;
    __nv_bfloat16* vt;
    int pos0, n_tokens, S_pad, R, R_pad;
    float inv_freq[HD / 2];
};

// Grid: blockIdx.y == 0 -> Q jobs, == 1 -> K/V jobs (64-row blocks).
// Q job: one thread per (token, head, pair) over S_pad rows.
// K/V job: a block handles 64 rows x one KV head; V is transposed through
// shared memory so the Vt writes are 128-byte rows.
__global__ void __launch_bounds__(256) prefill_prep_kernel(const __grid_constant__ PrepArgs A) {
    __shared__ float vtile[64][HD + 1];
    if (blockIdx.y == 0) {
        const int64_t total = static_cast<int64_t>(A.S_pad) * NH * (HD / 2);
        for (int64_t j = blockIdx.x * 256ll + threadIdx.x; j < total; j += 256ll * gridDim.x) {
            const int i = static_cast<int>(j / (NH * (HD / 2)));   // token
            const int rem = static_cast<int>(j % (NH * (HD / 2)));
            const int h = rem / (HD / 2), p = rem % (HD / 2);
            float y0 = 0.f, y1 = 0.f;
            if (i < A.n_tokens) {
                const float2 x = reinterpret_cast<const float2*>(A.q)[static_cast<size_t>(i) * NH * HD / 2 + rem];
                float sn, cs;
                sincosf(static_cast<float>(A.pos0 + i) * A.inv_freq[p], &sn, &cs);
                y0 = (x.x * cs - x.y * sn) * kQScale;
                y1 = (x.x * sn + x.y * cs) * kQScale;
            }
            reinterpret_cast<__nv_bfloat162*>(A.qb)[(static_cast<size_t>(h) * A.S_pad + i) * (HD / 2) + p] =
                __floats2bfloat162_rn(y0, y1);
        }
        return;
    }
    // K / V: blockIdx.x over (row block of 64, kv head)
    const int nblk = A.R_pad / 64;
    for (int b = blockIdx.x; b < nblk * NKV; b += gridDim.x) {
        const int kvh = b % NKV;
        const int r0 = (b / NKV) * 64;
        // each thread: 16 (row, pair) items of the 64 x 32 pairs
        for (int t = threadIdx.x; t < 64 * (HD / 2); t += 256) {
            const int rr = t / (HD / 2), p = t % (HD / 2);
            const int r = r0 + rr;
            float k0 = 0.f, k1 = 0.f, v0 = 0.f, v1 = 0.f;
            if (r < A.R) {
                const size_t off = static_cast<size_t>(r) * (NKV * HD) + kvh * HD + 2 * p;
                if (r < A.pos0) {
                    const float2 kk = *reinterpret_cast<const float2*>(A.kc + off);
                    const float2 vv = *reinterpret_cast<const float2*>(A.vc + off);
                    k0 = kk.x; k1 = kk.y; v0 = vv.x; v1 = vv.y;
                } else {
                    const int i = r - A.pos0;
                    const size_t src = static_cast<size_t>(i) * (NKV * HD) + kvh * HD + 2 * p;
                    const float2 kk = *reinterpret_cast<const float2*>(A.k + src);
                    const float2 vv = *reinterpret_cast<const float2*>(A.v + src);
                    float sn, cs;
                    sincosf(static_cast<float>(r) * A.inv_freq[p], &sn, &cs);
                    k0 = kk.x * cs - kk.y * sn;
                    k1 = kk.x * sn + kk.y * cs;
                    v0 = vv.x; v1 = vv.y;
                    *reinterpret_cast<float2*>(A.kc + off) = make_float2(k0, k1);  // append
                    *reinterpret_cast<float2*>(A.vc + off) = make_float2(v0, v1);
                }
            }
            reinterpret_cast<__nv_bfloat162*>(A.kb)[(static_cast<size_t>(kvh) * A.R_pad + r) * (HD / 2) + p] =
                __floats2bfloat162_rn(k0, k1);
            vtile[rr][2 * p] = v0;
            vtile[rr][2 * p + 1] = v1;
        }
        __syncthreads();
        // Vt[kvh][d][r0 .. r0+63]: thread -> (d, pair of rows)
        for (int t = threadIdx.x; t < HD * 32; t += 256) {
            const int d = t / 32, rp = t % 32;
            reinterpret_cast<__nv_bfloat162*>(A.vt)[((static_cast<size_t>(kvh) * HD + d) * A.R_pad + r0) / 2 + rp] =
                __floats2bfloat162_rn(vtile[2 * rp][d], vtile[2 * rp + 1][d]);
        }
        __syncthreads();
    }
}

struct AttnArgs {
    CUtensorMap tm_q;   // Qb as 2-D [NH*S_pad][64], box {64, 128}
    CUtensorMap tm_k;   // Kb as 2-D [NKV*R_pad][64], box {64, 128}
    CUtensorMap tm_vt;  // Vt as 2-D [NKV*64][R_pad], box {64, 64}
    float* out;         // [n_tokens][NH*HD]
    int pos0, n_tokens, S_pad, R_pad, n_qt;
    uint32_t* err;
};

// 97 KB: two CTAs fit on one SM (TMEM: 2 x 256 columns).
struct AttnSmem {
    __nv_bfloat16 q[BM * HD];          // 16 KB, SW128 K-major
    __nv_bfloat16 k[2][BN * HD];       // 2 stages x 16 KB
    __nv_bfloat16 vt[2][HD * 64];      // [kv half] 64 rows (d) x 64 kv: 2 x 8 KB
    __nv_bfloat16 p[2][BM * 64];       // [kv half] 128 rows x 64 kv: 2 x 16 KB
    uint64_t bar_q;
    uint64_t bar_k[2];
    uint64_t bar_v;
    uint64_t bar_s;
    uint64_t bar_o;
    uint32_t tmem_base;
};

constexpr uint32_t kTileBytesK = BN * HD * 2;        // 16 KB
constexpr uint32_t kTileBytesV = 2 * HD * 64 * 2;    // 16 KB
constexpr uint32_t kIdescS = idesc_bf16_f32(BM, BN);
constexpr uint32_t kIdescO = idesc_bf16_f32(BM, HD);

__device__ __forceinline__ void wait_or_flag(uint64_t* bar, uint32_t parity, uint32_t* err,
                                             uint32_t code) {
    if (!mbar_wait(bar, parity)) record_error(err, code);
}

__global__ void __launch_bounds__(ATTN_THREADS) prefill_attn_kernel(const __grid_constant__ AttnArgs A) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // SW128 atoms need 1024-byte aligned tiles (the launch adds 1 KB of slack)
    AttnSmem& S = *reinterpret_cast<AttnSmem*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    // heaviest query tiles first
    const int qt = A.n_qt - 1 - static_cast<int>(blockIdx.x) / NH;
    const int h = static_cast<int>(blockIdx.x) % NH;
    const int kvh = h / GQA;
    const int q0 = qt * BM;                                   // first query row (token index)
    const int last_tok = min(q0 + BM, A.n_tokens) - 1;
    const int n_kv = (A.pos0 + last_tok) / BN + 1;            // kv tiles needed
    const int first_pos = A.pos0 + q0;                        // position of row 0

    if (tid == 0) {
        mbar_init(&S.bar_q, 1);
        mbar_init(&S.bar_k[0], 1);
        mbar_init(&S.bar_k[1], 1);
        mbar_init(&S.bar_v, 1);
        mbar_init(&S.bar_s, 1);
        mbar_init(&S.bar_o, 1);
        fence_barrier_init();
        prefetch_tmap(&A.tm_q);
        prefetch_tmap(&A.tm_k);
        prefetch_tmap(&A.tm_vt);
    }
    if (warp == 0) {
        tmem_alloc(&S.tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    const uint32_t tmem_s = tmem;
    const uint32_t tmem_o = tmem + 128;

    // K tiles are double-buffered; the V^T tile is single-buffered and
    // reloaded as soon as the PV MMA that read it has completed.
    auto issue_k = [&](int j) {
        const int st = j & 1;
        mbar_arrive_expect_tx(&S.bar_k[st], kTileBytesK);
        tma_load_2d(S.k[st], &A.tm_k, 0, kvh * A.R_pad + j * BN, &S.bar_k[st]);
    };
    auto issue_v = [&](int j) {
        mbar_arrive_expect_tx(&S.bar_v, kTileBytesV);
        tma_load_2d(S.vt[0], &A.tm_vt, j * BN, kvh * HD, &S.bar_v);
        tma_load_2d(S.vt[1], &A.tm_vt, j * BN + 64, kvh * HD, &S.bar_v);
    };
    if (tid == 0) {
        mbar_arrive_expect_tx(&S.bar_q, BM * HD * 2);
        tma_load_2d(S.q, &A.tm_q, 0, h * A.S_pad + q0, &S.bar_q);
        issue_k(0);
        issue_v(0);
        if (n_kv > 1) issue_k(1);
    }

    const int row = tid;                      // query row of this thread (TMEM lane)
    const int my_pos = first_pos + row;       // its position (rows past n_tokens are discarded)
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    float o[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) o[d] = 0.f;

    const uint32_t q_addr = smem_u32(S.q);
    for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        // ---- S = Q K_j^T ----
        if (tid == 0) {
            if (j == 0) wait_or_flag(&S.bar_q, 0, A.err, kErrWaitFull);
            wait_or_flag(&S.bar_k[st], (j >> 1) & 1, A.err, kErrWaitFull);
            tc_fence_after();
            const uint32_t k_addr = smem_u32(S.k[st]);
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk)
                umma_bf16(tmem_s, sw128_desc(q_addr + 32 * kk), sw128_desc(k_addr + 32 * kk), kIdescS,
                          kk > 0);
            umma_commit(&S.bar_s);
        }
        wait_or_flag(&S.bar_s, j & 1, A.err, kErrWaitMma);
        tc_fence_after();

        // ---- online softmax on this thread's row ----
        float s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
            float tmp[32];
            tmem_ld32(tmem_s + lane_off + 32 * c, tmp);
#pragma unroll
            for (int i = 0; i < 32; ++i) s[32 * c + i] = tmp[i];
        }
        tmem_wait_ld();
        const int kv0 = j * BN;
        float mt = -INFINITY;
        if (kv0 + BN - 1 > my_pos) {
#pragma unroll
            for (int i = 0; i < BN; ++i)
                if (kv0 + i > my_pos) s[i] = -INFINITY;
        }
#pragma unroll
        for (int i = 0; i < BN; ++i) mt = fmaxf(mt, s[i]);
        const float m_new = fmaxf(m_run, mt);
        const float alpha = (m_run == -INFINITY) ? 0.f : exp2f((m_run - m_new) * kLog2e);
        const float mb = m_new * kLog2e;
        float lsum = 0.f;
        // P (bf16) into the swizzled K-major tile: row `row`, kv column c.
        unsigned char* prow0 = reinterpret_cast<unsigned char*>(S.p[0]) + row * 128;
        unsigned char* prow1 = reinterpret_cast<unsigned char*>(S.p[1]) + row * 128;
#pragma unroll
        for (int ch = 0; ch < BN / 8; ++ch) {   // 16 chunks of 8 kv columns (16 bytes)
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float p0 = exp2f(fmaf(s[8 * ch + 2 * e], kLog2e, -mb));
                const float p1 = exp2f(fmaf(s[8 * ch + 2 * e + 1], kLog2e, -mb));
                const __nv_bfloat162 b = __floats2bfloat162_rn(p0, p1);
                const float2 bf = __bfloat1622float2(b);
                lsum += bf.x + bf.y;
                w[e] = *reinterpret_cast<const uint32_t*>(&b);
            }
            const int blk = ch >> 3, cc = ch & 7;
            unsigned char* dst = (blk ? prow1 : prow0) + ((cc ^ (row & 7)) << 4);
            *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l_run = l_run * alpha + lsum;
        m_run = m_new;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();

        // ---- O_j = P V_j ----
        if (tid == 0) {
            wait_or_flag(&S.bar_v, j & 1, A.err, kErrWaitFull);
            tc_fence_after();
            const uint32_t p_addr = smem_u32(S.p[0]);
            const uint32_t v_addr = smem_u32(S.vt[0]);
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
                const uint32_t blk = kk >> 2, off = (kk & 3) * 32;
                umma_bf16(tmem_o, sw128_desc(p_addr + blk * (BM * 64 * 2) + off),
                          sw128_desc(v_addr + blk * (HD * 64 * 2) + off), kIdescO, kk > 0);
            }
            umma_commit(&S.bar_o);
        }
        wait_or_flag(&S.bar_o, j & 1, A.err, kErrWaitMma);
        tc_fence_after();
        // K stage st and the V^T buffer are free once the PV MMA finished
        if (tid == 0) {
            if (j + 1 < n_kv) issue_v(j + 1);
            if (j + 2 < n_kv) issue_k(j + 2);
        }
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
            float tmp[32];
            tmem_ld32(tmem_o + lane_off + 32 * c, tmp);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[32 * c + i] = fmaf(o[32 * c + i], alpha, tmp[i]);
        }
        tc_fence_before();
        __syncthreads();   // S / O_j TMEM and the P buffer may be reused
    }

    // ---- epilogue: out[token][h][:] = O / l ----
    const int tok = q0 + row;
    if (tok < A.n_tokens) {
        const float inv = 1.0f / l_run;
        float4* dst = reinterpret_cast<float4*>(A.out + static_cast<size_t>(tok) * NH * HD + h * HD);
#pragma unroll
        for (int d = 0; d < HD / 4; ++d)
            dst[d] = make_float4(o[4 * d] * inv, o[4 * d + 1] * inv, o[4 * d + 2] * inv, o[4 * d + 3] * inv);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---- host: tensor maps ------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

cudaError_t get_encoder(EncodeTiledFn* fn) {
    static EncodeTiledFn cached = nullptr;
    static std::once_flag once;
    static cudaError_t status = cudaSuccess;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (status == cudaSuccess && q != cudaDriverEntryPointSuccess) status = cudaErrorNotSupported;
        cached = reinterpret_cast<EncodeTiledFn>(p);
    });
    *fn = cached;
    return status;
}

// 2-D bf16 map over a row-major [rows][cols] array, box {64, box_rows},
// 128-byte swizzle (the UMMA K-major SW128 layout).
cudaError_t make_map(CUtensorMap* m, void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
    EncodeTiledFn enc = nullptr;
    cudaError_t e = get_encoder(&enc);
    if (e != cudaSuccess) return e;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

size_t prefill_workspace_bytes(int n_tokens, int pos0) {
    if (n_tokens <= 0 || pos0 < 0) return 0;
    return layout_for(n_tokens, pos0).total;
}

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream) {
    const Layout L = layout_for(a.n_tokens, a.pos0);
    unsigned char* ws = static_cast<unsigned char*>(a.workspace);
    PrepArgs p{};
    p.q = a.q;
    p.k = a.k;
    p.v = a.v;
    p.kc = a.key_cache + static_cast<size_t>(a.layer) * a.n_ctx * kRowFloats;
    p.vc = a.value_cache + static_cast<size_t>(a.layer) * a.n_ctx * kRowFloats;
    p.qb = reinterpret_cast<__nv_bfloat16*>(ws + L.qb_off);
    p.kb = reinterpret_cast<__nv_bfloat16*>(ws + L.kb_off);
    p.vt = reinterpret_cast<__nv_bfloat16*>(ws + L.vt_off);
    p.pos0 = a.pos0;
    p.n_tokens = a.n_tokens;
    p.S_pad = L.S_pad;
    p.R = L.R;
    p.R_pad = L.R_pad;
    for (int i = 0; i < HD / 2; ++i) p.inv_freq[i] = a.inv_freq[i];
    {
        const int64_t qjobs = static_cast<int64_t>(L.S_pad) * NH * (HD / 2);
        const int gx = static_cast<int>(std::min<int64_t>((qjobs + 255) / 256, 148 * 8));
        const int kvblocks = (L.R_pad / 64) * NKV;
        dim3 grid(std::max(gx, std::min(kvblocks, 148 * 8)), 2);
        prefill_prep_kernel<<<grid, 256, 0, stream>>>(p);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    AttnArgs t{};
    cudaError_t e = make_map(&t.tm_q, p.qb, HD, static_cast<uint64_t>(NH) * L.S_pad, BM);
    if (e != cudaSuccess) return e;
    e = make_map(&t.tm_k, p.kb, HD, static_cast<uint64_t>(NKV) * L.R_pad, BN);
    if (e != cudaSuccess) return e;
    e = make_map(&t.tm_vt, p.vt, static_cast<uint64_t>(L.R_pad), static_cast<uint64_t>(NKV) * HD, 64);
    if (e != cudaSuccess) return e;
    t.out = a.out;
    t.pos0 = a.pos0;
    t.n_tokens = a.n_tokens;
    t.S_pad = L.S_pad;
    t.R_pad = L.R_pad;
    t.n_qt = L.S_pad / BM;
    t.err = a.err;
    const int smem = static_cast<int>(sizeof(AttnSmem)) + 1024;
    static int configured_device = -1;
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (configured_device != dev) {
        e = cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured_device = dev;
    }
    prefill_attn_kernel<<<t.n_qt * NH, ATTN_THREADS, smem, stream>>>(t);
    return cudaGetLastError();
}

}  // namespace tle
