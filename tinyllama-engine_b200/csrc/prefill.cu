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
//  2. prefill_attn_kernel: persistent, one CTA per SM walking work items
//     (128-query tile, pair of query heads of one KV head), heaviest first in
//     snake order.  TMA (SWIZZLE_128B, no multicast) loads each item's two Q
//     tiles (double-buffered across items) and a 4-stage ring of 128-row K /
//     V^T tiles; one warp per head issues S = Q K^T (M=128, N=128, K=64) into
//     TMEM and O += P V (M=128, N=64, K=128, P read from TMEM); 128 threads
//     per head (one per query row) read S back, apply the causal mask and an
//     fp32 online softmax with a lazy rescale, and write P (bf16) to TMEM.
//     The next item's first scores are computed during this item's epilogue,
//     which stages O through the dead Q buffer for coalesced stores.  Q, K,
//     V and P enter the MMA as bf16 with fp32 accumulation (the north-star
//     prefill contract, tolerance 2e-2).  Both kernels are templates on the
//     16-bit type: the batched prompt (gemm.cu) runs them with fp16
//     operands, 3 more significand bits, because there the attention
//     output of one layer feeds the next (|q/8|, |k|, |v| and P <= 2^8 stay
//     far inside fp16's range for this model family).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
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
constexpr int ATTN_THREADS = 384;
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
    uint16_t* vt;         // bf16 bits
    int pos0, n_tokens, S_pad, R, R_pad;
    float inv_freq[HD / 2];
};

constexpr int kPrepThreads = 256;
static_assert(kPrepThreads == NKV * HD, "the V^T writer maps one thread to one (kv head, d) row");
constexpr int kPrepTokensPerBlock = kPrepThreads / 32;  // one token per warp
constexpr int kVtRows = 8;                               // rows per transpose block
constexpr int kVtPitch = NKV * HD + 8;                   // bf16 pitch of the transpose tile

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&b);
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}
// The 16-bit operand type of one instantiation: bf16 (tle_prefill) or fp16
// (the batched prompt, whose errors compound over layers).
template <bool F16>
__device__ __forceinline__ uint32_t pack16(float lo, float hi) {
    if constexpr (F16) return pack_f16(lo, hi);
    else return pack_bf16(lo, hi);
}

// blockIdx.y == 0: one token per warp, lane = rotation pair p.  One sincosf
//   per (token, pair) serves the 32 query heads and 4 key heads: rotated
//   q * 1/8 -> Qb, rotated k -> cache (append) and Kb.  Token slots in
//   [n_tokens, S_pad) zero their Qb rows.
// blockIdx.y == 1: 32 rows x all 4 KV heads: V rows (cache prefix, new
//   tokens, zero pad) are transposed through shared memory into Vt, and the
//   new tokens' v rows are appended to the cache; Kb rows of the cache prefix
//   (bf16 of the cached rotated k) and of the pad (zero).
template <bool F16>
__global__ void __launch_bounds__(kPrepThreads, 3) prefill_prep_kernel(const __grid_constant__ PrepArgs A) {
    __shared__ __align__(16) uint16_t vtile[kVtRows * kVtPitch];   // bf16 bits
    // The attention launch may start now (programmatic dependent launch): it
    // sets up its barriers and TMEM while this grid runs, and its TMA
    // producer waits for this grid to complete before loading the operands.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // This grid is itself a programmatic dependent of the previous kernel on
    // the stream (the producer of q, k and v): nothing is read before it ends.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (blockIdx.y == 0) {
        const int i = blockIdx.x * kPrepTokensPerBlock + warp;  // token
        if (i >= A.S_pad) return;
        uint32_t* qb32 = reinterpret_cast<uint32_t*>(A.qb);
        if (i >= A.n_tokens) {
#pragma unroll 4
            for (int h = 0; h < NH; ++h) qb32[(static_cast<size_t>(h) * A.S_pad + i) * (HD / 2) + lane] = 0u;
            return;
        }
        const int pos = A.pos0 + i;
        float sn, cs;
        sincosf(static_cast<float>(pos) * A.inv_freq[lane], &sn, &cs);
        // Every load of the token first (36 in flight per lane), then the
        // stores: loads placed after stores could not be hoisted above them.
        // (The v row is appended by the V^T role, which reads it anyway.)
        const float2* qs = reinterpret_cast<const float2*>(A.q + static_cast<size_t>(i) * NH * HD);
        const float2* ks = reinterpret_cast<const float2*>(A.k + static_cast<size_t>(i) * NKV * HD);
        float2 xq[NH], xk[NKV];
#pragma unroll
        for (int h = 0; h < NH; ++h) xq[h] = qs[h * (HD / 2) + lane];
#pragma unroll
        for (int g = 0; g < NKV; ++g) xk[g] = ks[g * (HD / 2) + lane];
#pragma unroll
        for (int h = 0; h < NH; ++h) {
            const float2 x = xq[h];
            qb32[(static_cast<size_t>(h) * A.S_pad + i) * (HD / 2) + lane] =
                pack16<F16>((x.x * cs - x.y * sn) * kQScale, (x.x * sn + x.y * cs) * kQScale);
        }
        float2* kcr = reinterpret_cast<float2*>(A.kc + static_cast<size_t>(pos) * NKV * HD);
        uint32_t* kb32 = reinterpret_cast<uint32_t*>(A.kb);
#pragma unroll
        for (int g = 0; g < NKV; ++g) {
            const float2 x = xk[g];
            const float2 y = make_float2(x.x * cs - x.y * sn, x.x * sn + x.y * cs);
            kcr[g * (HD / 2) + lane] = y;                                     // append (ops.cpp:1370)
            kb32[(static_cast<size_t>(g) * A.R_pad + pos) * (HD / 2) + lane] = pack16<F16>(y.x, y.y);
        }
        return;
    }
    // ---- V^T and the Kb rows not written by the token role ----
    const int r0 = blockIdx.x * kVtRows;
    if (r0 >= A.R_pad) return;
    constexpr int kVec = NKV * HD / 4;                       // float4 per row (64)
    constexpr int kPerThread = kVtRows * kVec / kPrepThreads; // 8
    float4 vv[kPerThread];
#pragma unroll
    for (int u = 0; u < kPerThread; ++u) {                   // all loads in flight
        const int t = threadIdx.x + u * kPrepThreads;
        const int rr = t / kVec, c4 = t % kVec;
        const int r = r0 + rr;
        vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < A.pos0)
            vv[u] = reinterpret_cast<const float4*>(A.vc + static_cast<size_t>(r) * NKV * HD)[c4];
        else if (r < A.R)
            vv[u] = reinterpret_cast<const float4*>(A.v + static_cast<size_t>(r - A.pos0) * NKV * HD)[c4];
    }
#pragma unroll
    for (int u = 0; u < kPerThread; ++u) {
        const int t = threadIdx.x + u * kPrepThreads;
        const int rr = t / kVec, c4 = t % kVec;
        const int r = r0 + rr;
        if (r >= A.pos0 && r < A.R)   // append v of the new tokens (ops.cpp:1371)
            reinterpret_cast<float4*>(A.vc + static_cast<size_t>(r) * NKV * HD)[c4] = vv[u];
        *reinterpret_cast<uint2*>(&vtile[rr * kVtPitch + 4 * c4]) =
            make_uint2(pack16<F16>(vv[u].x, vv[u].y), pack16<F16>(vv[u].z, vv[u].w));
        // Kb rows outside [pos0, R): bf16 of the cached prefix, zero pad
        if (r < A.pos0 || r >= A.R) {
            float4 kk = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < A.pos0) kk = reinterpret_cast<const float4*>(A.kc + static_cast<size_t>(r) * NKV * HD)[c4];
            const int g = c4 / (HD / 4), d4 = c4 % (HD / 4);
            *reinterpret_cast<uint2*>(A.kb + (static_cast<size_t>(g) * A.R_pad + r) * HD + 4 * d4) =
                make_uint2(pack16<F16>(kk.x, kk.y), pack16<F16>(kk.z, kk.w));
        }
    }
    __syncthreads();
    // thread -> one (kv head, d) row of Vt: kVtRows consecutive kv positions
    {
        const int gd = threadIdx.x;  // 0 .. NKV*HD-1
        uint32_t w[kVtRows / 2];
#pragma unroll
        for (int e = 0; e < kVtRows / 2; ++e) {
            w[e] = static_cast<uint32_t>(vtile[(2 * e) * kVtPitch + gd]) |
                   (static_cast<uint32_t>(vtile[(2 * e + 1) * kVtPitch + gd]) << 16);
        }
        uint4* dst = reinterpret_cast<uint4*>(A.vt + static_cast<size_t>(gd) * A.R_pad + r0);
#pragma unroll
        for (int e = 0; e < kVtRows / 8; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
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

// Warp roles of prefill_attn_kernel (384 threads = 3 warpgroups, one CTA/SM):
//   warpgroup 0: warp 0 issues TMA loads, warps 1 and 2 issue tcgen05.mma
//                for query head h0 and h0+1, warp 3 idle (56 registers each
//                after setmaxnreg.dec);
//   warpgroups 1, 2: softmax of query head h0 / h0+1 (224 registers each),
//                one TMEM lane (= query row) per thread, all 128 columns.
// Register split: 384 x 168 at launch = 128 x 56 + 256 x 224.
constexpr int KSTAGES = 4;
constexpr int kRegsControl = 56;
constexpr int kRegsSoftmax = 224;
constexpr int kLaunchRegs = 168;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= ATTN_THREADS * kLaunchRegs,
              "setmaxnreg split exceeds the launch register budget");

// TMEM columns (512, the whole SM): S_i = Q_i K^T (fp32, 128 columns each),
// P_i = softmax numerators (bf16 pairs, 64 columns), O_i = P V (fp32, 64).
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColP0 = 256, kColP1 = 320, kColO0 = 384, kColO1 = 448;
constexpr uint32_t TMEM_COLS2 = 512;
// Lazy rescale: the running reference max only moves when the row max grows
// by more than 8 (log2 units), so O in TMEM is rescaled rarely; P <= 2^8.
constexpr float kRescaleThreshold = 8.0f;

struct AttnSmem {
    __nv_bfloat16 q[2][2][BM * HD];        // [item parity][head] 16 KB each, SW128 K-major
    __nv_bfloat16 k[KSTAGES][BN * HD];     // 16 KB per stage
    __nv_bfloat16 vt[KSTAGES][2][HD * 64]; // 16 KB per stage (two 64-kv halves)
    uint64_t bar_q[2];                     // Q tiles of an item landed
    uint64_t q_free[2];                    // Q buffer reusable: both heads' last S MMA of the
                                           // item done and its epilogue staging read back
    uint64_t kv_full[KSTAGES];
    uint64_t kv_empty[KSTAGES];
    uint64_t s_full[2];
    uint64_t s_free[2];
    uint64_t p_full[2];
    uint64_t p_free[2];
    uint32_t tmem_base;
};

constexpr uint32_t kTileBytesK = BN * HD * 2;        // 16 KB
constexpr uint32_t kTileBytesV = 2 * HD * 64 * 2;    // 16 KB
constexpr uint32_t kIdescS = idesc_bf16_f32(BM, BN);
constexpr uint32_t kIdescO = idesc_bf16_f32(BM, HD);

// 2^x on the SFU (MUFU.EX2, flush-to-zero; 2^-inf = 0).
__device__ __forceinline__ float ex2_sfu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// sm_100 packed fp32x2 arithmetic (two lanes of work per instruction).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// 2^x for a pair, on the FMA/ALU pipes, for a share of the elements so that the SFU is not
// the only exponential unit: round-to-nearest split x = n + f (f in
// [-1/2, 1/2]) with the 1.5*2^23 shifter, 2^f by a cubic fitted to 2^f on
// [-1/2, 1/2] (least squares on relative error, Chebyshev nodes, Lawson
// reweighting; max relative error 7.5e-5, far below the bf16 rounding of P),
// and n added to the exponent field.  x is clamped at -126 so masked (-inf)
// scores give ~1e-38 instead of a denormal.
__device__ __forceinline__ void ex2_poly2(uint64_t x2, float& r0, float& r1) {
    float x0, x1;
    f2_split(x2, x0, x1);
    x2 = f2(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
    const uint64_t sh = f2(12582912.0f, 12582912.0f);
    const uint64_t nsh = f2(-12582912.0f, -12582912.0f);
    const uint64_t t = fadd2(x2, sh);
    const uint64_t n = fadd2(t, nsh);
    const uint64_t f = ffma2(n, f2(-1.0f, -1.0f), x2);
    uint64_t p = ffma2(f2(0.0551716648f, 0.0551716648f), f, f2(0.2426111251f, 0.2426111251f));
    p = ffma2(p, f, f2(0.6932609677f, 0.6932609677f));
    p = ffma2(p, f, f2(0.9999280572f, 0.9999280572f));
    float t0, t1, p0, p1;
    f2_split(t, t0, t1);
    f2_split(p, p0, p1);
    const int kSh = __float_as_int(12582912.0f);
    r0 = __int_as_float(__float_as_int(p0) + ((__float_as_int(t0) - kSh) << 23));
    r1 = __int_as_float(__float_as_int(p1) + ((__float_as_int(t1) - kSh) << 23));
}

// Bounded wait; after the first expiry in a thread every later wait of that
// thread returns at once, so a broken pipeline unwinds in ~one timeout.
__device__ __forceinline__ void wait_or_flag(uint64_t* bar, uint32_t parity, uint32_t* err,
                                             uint32_t code, bool& failed) {
    if (failed) return;
    if (!mbar_wait(bar, parity)) {
        record_error(err, code);
        failed = true;
    }
}

// Work items: (128-query tile, pair of query heads of one KV head), numbered
// heaviest query tile first.  The persistent CTAs take them in snake order
// (round r: CTA c takes r G + c for even r, r G + G - 1 - c for odd r), which
// evens out the causal tile counts.
struct Item {
    int h0, kvh, q0, n_kv;
};
__device__ __forceinline__ int item_index(int k, int c, int G) {
    return k * G + ((k & 1) ? G - 1 - c : c);
}
__device__ __forceinline__ Item item_at(const AttnArgs& A, int idx) {
    Item it;
    const int qt = A.n_qt - 1 - idx / (NH / 2);
    it.h0 = 2 * (idx % (NH / 2));
    it.kvh = it.h0 / GQA;
    it.q0 = qt * BM;
    const int last_tok = min(it.q0 + BM, A.n_tokens) - 1;
    it.n_kv = (A.pos0 + last_tok) / BN + 1;
    return it;
}

template <bool F16>
__global__ void __launch_bounds__(ATTN_THREADS, 1) prefill_attn_kernel(const __grid_constant__ AttnArgs A) {
    constexpr uint32_t kIdS = F16 ? idesc_f16_f32(BM, BN) : kIdescS;
    constexpr uint32_t kIdO = F16 ? idesc_f16_f32(BM, HD) : kIdescO;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // SW128 atoms need 1024-byte aligned tiles (the launch adds 1 KB of slack)
    AttnSmem& S = *reinterpret_cast<AttnSmem*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int wg = warp >> 2;
    // the next kernel on the stream may be scheduled as this grid's CTAs
    // leave their SMs (it waits for this grid before reading its output)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int n_items = A.n_qt * (NH / 2);
    const int G = static_cast<int>(gridDim.x);
    const int cta = static_cast<int>(blockIdx.x);
    int my_items = 0;   // items of this CTA: k = 0 .. my_items-1
    while (item_index(my_items, cta, G) < n_items) ++my_items;

    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.bar_q[b], 1);
            mbar_init(&S.q_free[b], 2 + 8);   // a commit per head's MMA warp + the 8 softmax warps
        }
        for (int i = 0; i < KSTAGES; ++i) {
            mbar_init(&S.kv_full[i], 1);
            mbar_init(&S.kv_empty[i], 2);   // last PV of each head
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S.s_full[i], 1);
            mbar_init(&S.s_free[i], 4);   // one arrival per softmax warp of the head
            mbar_init(&S.p_full[i], 4);
            mbar_init(&S.p_free[i], 1);
        }
        fence_barrier_init();
        prefetch_tmap(&A.tm_q);
        prefetch_tmap(&A.tm_k);
        prefetch_tmap(&A.tm_vt);
    }
    if (warp == 0) {
        tmem_alloc(&S.tmem_base, TMEM_COLS2);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    bool failed = false;

    if (wg == 0) {
        regs_dealloc<kRegsControl>();
        if (warp == 0) {
            // ------------------------------ TMA producer ------------------------------
            // Qb, Kb and Vt are written by prefill_prep_kernel, the preceding
            // launch on the stream (no-op without programmatic dependent launch).
            asm volatile("griddepcontrol.wait;" ::: "memory");
            int ring = 0;   // K/V tiles issued so far (across items)
            for (int k = 0; k < my_items; ++k) {
                const Item it = item_at(A, item_index(k, cta, G));
                const int b = k & 1;
                // Q buffer b was last read by item k-2's S MMAs
                if (k >= 2) wait_or_flag(&S.q_free[b], ((k >> 1) - 1) & 1, A.err, kErrWaitEmpty, failed);
                if (lane == 0) {
                    mbar_arrive_expect_tx(&S.bar_q[b], 2 * BM * HD * 2);
                    tma_load_2d(S.q[b][0], &A.tm_q, 0, it.h0 * A.S_pad + it.q0, &S.bar_q[b]);
                    tma_load_2d(S.q[b][1], &A.tm_q, 0, (it.h0 + 1) * A.S_pad + it.q0, &S.bar_q[b]);
                }
                for (int j = 0; j < it.n_kv; ++j, ++ring) {
                    const int st = ring % KSTAGES;
                    wait_or_flag(&S.kv_empty[st], ((ring / KSTAGES) & 1) ^ 1, A.err, kErrWaitEmpty, failed);
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&S.kv_full[st], kTileBytesK + kTileBytesV);
                        tma_load_2d(S.k[st], &A.tm_k, 0, it.kvh * A.R_pad + j * BN, &S.kv_full[st]);
                        tma_load_2d(S.vt[st][0], &A.tm_vt, j * BN, it.kvh * HD, &S.kv_full[st]);
                        tma_load_2d(S.vt[st][1], &A.tm_vt, j * BN + 64, it.kvh * HD, &S.kv_full[st]);
                    }
                    __syncwarp();
                }
            }
        } else if (warp == 1 || warp == 2) {
            // ------------------------------ MMA issuers --------------------------------
            // One issuing warp per query head, so the two heads' pipelines do
            // not wait on each other: head i issues S_i of its next tile as
            // soon as its softmax has read the current one (across item
            // boundaries too, so the next item's first scores are computed
            // during this item's epilogue), and O_i += P_i V as soon as P_i is
            // in TMEM.  A K/V stage is released when both heads' last readers
            // of it have committed (kv_empty counts 2 arrivals); a Q buffer
            // when both heads' last S MMA of the item has (q_free, 2).
            const int i = warp - 1;
            const uint64_t dk0 = sw128_desc(smem_u32(S.k[0]));
            const uint64_t dv0 = sw128_desc(smem_u32(S.vt[0][0]));
            constexpr uint64_t kStageK = (BN * HD * 2) >> 4;        // stage stride, descriptor units
            constexpr uint64_t kStageV = (2 * HD * 64 * 2) >> 4;
            constexpr uint64_t kHalfV = (HD * 64 * 2) >> 4;         // 8 KB in descriptor units
            const uint32_t tS = tmem + (i ? kColS1 : kColS0);
            const uint32_t tP = tmem + (i ? kColP1 : kColP0);
            const uint32_t tO = tmem + (i ? kColO1 : kColO0);
            // S_i of global tile g (item k, tile n; the stage of a tile is its
            // global index: the producer walks the same sequence)
            auto issue_s = [&](int g, int k, int n, int n_kv) {
                const int st = g % KSTAGES;
                const int b = k & 1;
                if (n == 0) wait_or_flag(&S.bar_q[b], (k >> 1) & 1, A.err, kErrWaitFull, failed);
                wait_or_flag(&S.kv_full[st], (g / KSTAGES) & 1, A.err, kErrWaitFull, failed);
                if (g > 0) wait_or_flag(&S.s_free[i], (g - 1) & 1, A.err, kErrWaitMma, failed);
                tc_fence_after();
                if (elect_one()) {
                    const uint64_t dq = sw128_desc(smem_u32(S.q[b][i]));
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        umma_bf16(tS, dq + 2 * kk, dk0 + st * kStageK + 2 * kk, kIdS, kk > 0);
                    umma_commit(&S.s_full[i]);
                    if (n == n_kv - 1) umma_commit(&S.q_free[b]);   // last read of Q buffer b
                }
                __syncwarp();
            };
            auto issue_pv = [&](int g, int n) {  // O_i (+)= P_i V of global tile g (tile n of its item)
                const int st = g % KSTAGES;
                wait_or_flag(&S.p_full[i], g & 1, A.err, kErrWaitMma, failed);
                tc_fence_after();
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < BN / 16; ++kk)
                        umma_bf16_tmem_a(tO, tP + 8 * kk,
                                         dv0 + st * kStageV + (kk >> 2) * kHalfV + 2 * (kk & 3), kIdO,
                                         (n > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&S.p_free[i]);
                    umma_commit(&S.kv_empty[st]);
                }
                __syncwarp();
            };
            if (my_items > 0) {
                int k = 0, n = 0, g = 0;
                Item it = item_at(A, item_index(0, cta, G));
                issue_s(0, 0, 0, it.n_kv);
                for (;;) {
                    // the tile after (k, n): scores first, then this tile's PV
                    int k2 = k, n2 = n + 1;
                    Item it2 = it;
                    if (n2 == it.n_kv) {
                        k2 = k + 1;
                        n2 = 0;
                        if (k2 < my_items) it2 = item_at(A, item_index(k2, cta, G));
                    }
                    const bool more = k2 < my_items;
                    if (more) issue_s(g + 1, k2, n2, it2.n_kv);
                    issue_pv(g, n);
                    if (!more) break;
                    k = k2;
                    n = n2;
                    it = it2;
                    ++g;
                }
            }
        }
    } else {
        // ------------------------------ softmax ------------------------------------
        regs_alloc<kRegsSoftmax>();
        const int i = wg - 1;                       // which query head of the pair
        const int row = tid - 128 * wg;             // query row = TMEM lane
        const uint32_t lanes = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lanes + (i ? kColS1 : kColS0);
        const uint32_t tP = tmem + lanes + (i ? kColP1 : kColP0);
        const uint32_t tO = tmem + lanes + (i ? kColO1 : kColO0);
        int g = 0;   // global tile index of this head (barrier phases run across items)
        for (int k = 0; k < my_items; ++k) {
            const Item it = item_at(A, item_index(k, cta, G));
            const int q0 = it.q0;
            const int n_kv = it.n_kv;
            const int my_pos = A.pos0 + q0 + row;
            float m_ref = -INFINITY;   // reference max, log2 units
            float l_run = 0.f;
            for (int j = 0; j < n_kv; ++j, ++g) {
                wait_or_flag(&S.s_full[i], g & 1, A.err, kErrWaitMma, failed);
                tc_fence_after();
                float s[BN];
#pragma unroll
                for (int c = 0; c < BN / 32; ++c) {
                    float tmp[32];
                    tmem_ld32(tS + 32 * c, tmp);
#pragma unroll
                    for (int e = 0; e < 32; ++e) s[32 * c + e] = tmp[e];
                }
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.s_free[i]);   // the MMA may overwrite S_i

                const int kv0 = j * BN;
                if (kv0 + BN - 1 > my_pos) {
#pragma unroll
                    for (int e = 0; e < BN; ++e)
                        if (kv0 + e > my_pos) s[e] = -INFINITY;
                }
                // row max as 16 independent 8-element chains, then a 3-input tree
                float mc[16];
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    float m = fmax3(s[8 * c], s[8 * c + 1], s[8 * c + 2]);
                    m = fmax3(m, s[8 * c + 3], s[8 * c + 4]);
                    m = fmax3(m, s[8 * c + 5], s[8 * c + 6]);
                    mc[c] = fmaxf(m, s[8 * c + 7]);
                }
#pragma unroll
                for (int c = 0; c < 5; ++c) mc[c] = fmax3(mc[3 * c], mc[3 * c + 1], mc[3 * c + 2]);
                const float mt = fmax3(fmax3(mc[0], mc[1], mc[2]), fmax3(mc[3], mc[4], mc[15]), -INFINITY) * kLog2e;
                float alpha = 1.f;
                const bool move = mt > m_ref + kRescaleThreshold;
                if (move) {
                    alpha = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - mt);
                    m_ref = mt;
                }
                // P = 2^(s*log2e - m_ref) in fp32 (5 pairs in 16 on the FMA
                // pipe, the rest on the SFU: measured best of 0 .. 50 %),
                // packed to bf16 pairs; fp32 row sum.
                const uint64_t l2e2 = f2(kLog2e, kLog2e);
                const uint64_t negm2 = f2(-m_ref, -m_ref);
                uint32_t pk[BN / 2];
                uint64_t lsum2[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
                // pass 1: all exponent arguments (in place of the scores)
#pragma unroll
                for (int e = 0; e < BN / 2; ++e)
                    f2_split(ffma2(f2(s[2 * e], s[2 * e + 1]), l2e2, negm2), s[2 * e], s[2 * e + 1]);
                // pass 2: exponentials, SFU and FMA-pipe pairs interleaved
#pragma unroll
                for (int e = 0; e < BN / 2; ++e) {
                    float p0, p1;
                    if ((e & 15) == 2 || (e & 15) == 5 || (e & 15) == 7 || (e & 15) == 10 || (e & 15) == 13) {
                        ex2_poly2(f2(s[2 * e], s[2 * e + 1]), p0, p1);
                    } else {
                        p0 = ex2_sfu(s[2 * e]);
                        p1 = ex2_sfu(s[2 * e + 1]);
                    }
                    s[2 * e] = p0;
                    s[2 * e + 1] = p1;
                }
                // pass 3: row sum and bf16 packing
#pragma unroll
                for (int e = 0; e < BN / 2; ++e) {
                    lsum2[e & 3] = fadd2(lsum2[e & 3], f2(s[2 * e], s[2 * e + 1]));
                    pk[e] = pack16<F16>(s[2 * e], s[2 * e + 1]);
                }
                float lsum0, lsum1;
                f2_split(fadd2(fadd2(lsum2[0], lsum2[1]), fadd2(lsum2[2], lsum2[3])), lsum0, lsum1);
                l_run = l_run * alpha + (lsum0 + lsum1);
                // P_i and O_i may be touched once the previous PV MMA is done
                if (j > 0) {
                    wait_or_flag(&S.p_free[i], (g - 1) & 1, A.err, kErrWaitMma, failed);
                    tc_fence_after();
                    if (__any_sync(0xffffffffu, move)) {
#pragma unroll
                        for (int c = 0; c < HD / 32; ++c) {
                            float o[32];
                            tmem_ld32(tO + 32 * c, o);
                            tmem_wait_ld();
                            uint32_t ob[32];
#pragma unroll
                            for (int e = 0; e < 32; ++e) ob[e] = __float_as_uint(o[e] * alpha);
                            tmem_st32(tO + 32 * c, ob);
                        }
                    }
                }
                tmem_st32(tP, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
                tmem_st32(tP + 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.p_full[i]);
            }
            // ---- epilogue: out[token][h][:] = O / l (the wait also frees P and
            // O for the next item's first tile).  O goes through this head's
            // Q buffer (its last reader, the item's last S MMA, finished
            // before S was read) so the global stores are coalesced: each
            // warp stages its own 32 rows, 32 columns at a time, 16-byte
            // chunk j of row r at chunk j ^ (r & 7) (conflict-free both ways),
            // then writes 4 rows x 128 B per store instruction. ----
            wait_or_flag(&S.p_free[i], (g - 1) & 1, A.err, kErrWaitMma, failed);
            tc_fence_after();
            const float inv = 1.0f / l_run;
            float* stg = reinterpret_cast<float*>(S.q[k & 1][i]);   // [128 rows][32 floats]
            const int qd = warp & 3;
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                float o[32];
                tmem_ld32(tO + 32 * c, o);
                tmem_wait_ld();
#pragma unroll
                for (int jc = 0; jc < 8; ++jc)
                    *reinterpret_cast<float4*>(stg + row * 32 + 4 * (jc ^ (row & 7))) =
                        make_float4(o[4 * jc] * inv, o[4 * jc + 1] * inv, o[4 * jc + 2] * inv, o[4 * jc + 3] * inv);
                __syncwarp();
#pragma unroll
                for (int kq = 0; kq < 8; ++kq) {
                    const int rr = 32 * qd + 4 * kq + (lane >> 3);
                    const int jc = lane & 7;
                    const float4 v = *reinterpret_cast<const float4*>(stg + rr * 32 + 4 * (jc ^ (rr & 7)));
                    const int tok = q0 + rr;
                    if (tok < A.n_tokens)
                        *reinterpret_cast<float4*>(A.out + static_cast<size_t>(tok) * NH * HD + (it.h0 + i) * HD +
                                                   32 * c + 4 * jc) = v;
                }
                __syncwarp();
            }
            // the Q buffer is rewritten by a TMA load (async proxy) once q_free completes
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.q_free[k & 1]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS2);
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
cudaError_t make_map(CUtensorMap* m, void* base, uint64_t cols, uint64_t rows, uint32_t box_rows,
                     CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
    EncodeTiledFn enc = nullptr;
    cudaError_t e = get_encoder(&enc);
    if (e != cudaSuccess) return e;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, dtype, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

cudaError_t make_tmap_16b(CUtensorMap* m, void* base, uint64_t cols, uint64_t rows, uint32_t box_rows,
                          CUtensorMapDataType dtype) {
    return make_map(m, base, cols, rows, box_rows, dtype);
}

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
    p.vt = reinterpret_cast<uint16_t*>(ws + L.vt_off);
    p.pos0 = a.pos0;
    p.n_tokens = a.n_tokens;
    p.S_pad = L.S_pad;
    p.R = L.R;
    p.R_pad = L.R_pad;
    for (int i = 0; i < HD / 2; ++i) p.inv_freq[i] = a.inv_freq[i];
    {
        // a programmatic dependent of the previous kernel (it waits for it
        // before its first load), so its launch overlaps that kernel's tail
        const int gx = std::max((L.S_pad + kPrepTokensPerBlock - 1) / kPrepTokensPerBlock, L.R_pad / kVtRows);
        cudaLaunchConfig_t pc{};
        pc.gridDim = dim3(gx, 2);
        pc.blockDim = dim3(kPrepThreads);
        pc.stream = stream;
        cudaLaunchAttribute pa[1];
        pa[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        pa[0].val.programmaticStreamSerializationAllowed = 1;
        pc.attrs = pa;
        pc.numAttrs = 1;
        cudaError_t e = a.f16 ? cudaLaunchKernelEx(&pc, prefill_prep_kernel<true>, p)
                              : cudaLaunchKernelEx(&pc, prefill_prep_kernel<false>, p);
        if (e != cudaSuccess) return e;
    }
    AttnArgs t{};
    const CUtensorMapDataType dt = a.f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    cudaError_t e = make_map(&t.tm_q, p.qb, HD, static_cast<uint64_t>(NH) * L.S_pad, BM, dt);
    if (e != cudaSuccess) return e;
    e = make_map(&t.tm_k, p.kb, HD, static_cast<uint64_t>(NKV) * L.R_pad, BN, dt);
    if (e != cudaSuccess) return e;
    e = make_map(&t.tm_vt, p.vt, static_cast<uint64_t>(L.R_pad), static_cast<uint64_t>(NKV) * HD, 64, dt);
    if (e != cudaSuccess) return e;
    t.out = a.out;
    t.pos0 = a.pos0;
    t.n_tokens = a.n_tokens;
    t.S_pad = L.S_pad;
    t.R_pad = L.R_pad;
    t.n_qt = L.S_pad / BM;
    t.err = a.err;
    const int smem = static_cast<int>(sizeof(AttnSmem)) + 1024;
    static PerDeviceOnce once;
    static int sm_count_of[kMaxDevices];
    e = once.run([&](int dev) {
        cudaError_t r0 = cudaDeviceGetAttribute(&sm_count_of[dev], cudaDevAttrMultiProcessorCount, dev);
        if (r0 != cudaSuccess) return r0;
        // setmaxnreg.inc waits until the block's launch registers cover the
        // split; refuse to launch (instead of hanging) if the compiled kernel
        // was given fewer registers than the split assumes.
        for (const void* fn : {reinterpret_cast<const void*>(prefill_attn_kernel<false>),
                               reinterpret_cast<const void*>(prefill_attn_kernel<true>)}) {
            cudaFuncAttributes fa{};
            cudaError_t r = cudaFuncGetAttributes(&fa, fn);
            if (r != cudaSuccess) return r;
            if (fa.numRegs < kLaunchRegs) return cudaErrorInvalidConfiguration;
            r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (r != cudaSuccess) return r;
        }
        return cudaSuccess;
    });
    if (e != cudaSuccess) return e;
    // Programmatic dependent launch: the attention grid may start while the
    // prep grid runs; only its TMA producer waits (griddepcontrol.wait).
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int n_sm = sm_count_of[dev];
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(std::min(t.n_qt * (NH / 2), n_sm));   // persistent: one CTA per SM
    cfg.blockDim = dim3(ATTN_THREADS);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (a.f16) return cudaLaunchKernelEx(&cfg, prefill_attn_kernel<true>, t);
    return cudaLaunchKernelEx(&cfg, prefill_attn_kernel<false>, t);
}

}  // namespace tle
