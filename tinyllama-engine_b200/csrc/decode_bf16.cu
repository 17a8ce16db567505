// decode_bf16.cu -- decode step over a bf16 KV cache (the reduced-precision
// cache variant of run_state.h:20-25), fused RoPE + append + attention for a
// batch of sequences.
//
// Reference semantics: rope() src/ops.cpp:1223-1281 then attention()
// src/ops.cpp:1317-1515 per sequence, with the cache rows stored as bf16:
// the appended row pos holds bf16(rotated k) and bf16(v) (round to nearest
// even), and every score and weighted sum reads the stored values.  The
// query and the softmax weights enter the tensor cores as bf16 with fp32
// accumulation, so the result agrees with the fp32 reference to bf16
// precision (2e-2, the prefill contract), not to the fp32 decode's 1e-4.
//
// Design: cache rows are 512 bytes (4 KV heads x 64 bf16).  CTA (c, s) takes
// chunk c (A.chunk rows) of sequence s and streams it in 64-row tiles of
// all four KV heads through a 3-stage shared-memory ring with 16-byte
// cp.async (16-byte chunks XOR-swizzled by row so the ldmatrix reads are
// conflict-free; rows past the chunk are zero-filled).  Warp w takes KV head
// g = w & 3 over keys [32 h, 32 h + 32) of every tile (h = w >> 2): S =
// Q_g K^T with mma.sync m16n8k16 (A = the 8 query heads of g, padded to 16
// rows; B = K rows via ldmatrix), an online softmax in the log2 domain, and
// O += P V with P re-packed from the S fragments as the A operand and V
// through ldmatrix.trans.  The two key halves of a head are folded in shared
// memory; a sequence of one chunk writes its output, otherwise the chunk
// writes (o / l, log-sum-exp) and merge_bf16_kernel combines the chunks.
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace tle {

namespace {

constexpr int BHD = kHeadDim;           // 64
constexpr int BNKV = kNHeadKv;          // 4
constexpr int BNH = kNHead;             // 32
constexpr int BROW = BNKV * BHD;        // 256 bf16 per cache row
constexpr int BTILE = 64;               // rows per tile
constexpr int BSTAGES = 3;
constexpr int BTHREADS = 256;
constexpr int kTileHalfs = BTILE * BROW;                 // bf16 per K (or V) tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct BfSmem {
    uint16_t k[BSTAGES][kTileHalfs];     // 32 KB per stage, swizzled 16-byte chunks
    uint16_t v[BSTAGES][kTileHalfs];
    uint16_t q[BNH * BHD];               // rotated q / 8, bf16
    float fold[BNKV][32][18];            // second key half: O (16 per lane), m, l
};

// Byte offset of 16-byte chunk c (0..31: KV head c / 8, dims 8 (c % 8)..)
// of tile row r: the chunk index within the head is XORed with r mod 8.
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
    return static_cast<uint32_t>(r * (BROW * 2) + (((c & ~7) | ((c ^ r) & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// D += A B for the m16n8k16 bf16 shape; rows 8-15 of A are zero here (a1 = a3 = 0).
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ float bf16_round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 16-byte cp.async, zero-filled when !valid (src is then any readable address).
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}

// A sequence as the kernel sees it: its position and where its rows are.
// Contiguous: row r of the layer at kc/vc + 256 r.  Paged: row r at page
// pages[r >> page_shift] of the pools (an id outside the pool is reported
// as 0x105 and its rows are neither read nor written).
template <bool PAGED>
struct BfSeqView {
    int pos;
    bool ok;
    uint16_t* kc;
    uint16_t* vc;
    const int32_t* pages;
};
template <bool PAGED>
__device__ __forceinline__ BfSeqView<PAGED> bf_seq(const BfArgs& A, int s) {
    BfSeqView<PAGED> v{};
    if (PAGED) {
        const tle_paged_seq_t ps = A.pseqs[s];
        v.pos = ps.pos;
        v.ok = ps.pos >= 0 && (static_cast<long long>(ps.n_pages) << A.page_shift) > ps.pos;
        v.pages = ps.pages;
        const size_t layer = static_cast<size_t>(A.layer) * A.pool_pages << A.page_shift;
        v.kc = static_cast<uint16_t*>(A.key_pool) + layer * BROW;
        v.vc = static_cast<uint16_t*>(A.value_pool) + layer * BROW;
    } else {
        const tle_seq_bf16_t sq = A.seqs[s];
        v.pos = sq.pos;
        v.ok = sq.pos >= 0 && sq.pos < sq.n_ctx;
        v.kc = static_cast<uint16_t*>(sq.key_cache) + static_cast<size_t>(A.layer) * sq.n_ctx * BROW;
        v.vc = static_cast<uint16_t*>(sq.value_cache) + static_cast<size_t>(A.layer) * sq.n_ctx * BROW;
        v.pages = nullptr;
    }
    return v;
}
// Element offset of row r from kc / vc; false (reported) for a bad page id.
template <bool PAGED>
__device__ __forceinline__ bool bf_row(const BfArgs& A, const BfSeqView<PAGED>& v, int r, size_t& off) {
    if (!PAGED) {
        off = static_cast<size_t>(r) * BROW;
        return true;
    }
    const int id = __ldg(v.pages + (r >> A.page_shift));
    if (static_cast<unsigned>(id) >= static_cast<unsigned>(A.pool_pages)) {
        record_error(A.err, kErrBadPage);
        return false;
    }
    off = ((static_cast<size_t>(id) << A.page_shift) | static_cast<size_t>(r & ((1 << A.page_shift) - 1))) * BROW;
    return true;
}

template <bool PAGED>
__global__ void __launch_bounds__(BTHREADS, 1) decode_bf16_kernel(const __grid_constant__ BfArgs A) {
    extern __shared__ __align__(128) unsigned char bf_raw[];
    BfSmem& S = *reinterpret_cast<BfSmem*>(bf_raw);
    // a programmatic dependent of the previous kernel (scheduled as it
    // drains); everything this kernel reads may be that kernel's output
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, s = blockIdx.y;
    const BfSeqView<PAGED> sq = bf_seq<PAGED>(A, s);
    const int L = sq.pos + 1;
    const int n_chunks = (L + A.chunk - 1) / A.chunk;
    // a record outside its cache (or page table), or longer than the
    // launch's max_rows, is reported and skipped (no access)
    if (!sq.ok || n_chunks > A.max_chunks) {
        if (c == 0 && tid == 0) record_error(A.err, kErrBadSeq);
        return;
    }
    const int r0 = c * A.chunk;
    if (r0 >= L) return;                                   // past the sequence's last chunk
    const int nrows = min(A.chunk, L - r0);
    const bool has_new = r0 + nrows == L;
    uint16_t* kc = sq.kc;
    uint16_t* vc = sq.vc;

    // q of sequence s: rotate (ops.cpp:1229-1260), x 1/8 (exact), bf16.
    // Thread t: pair t & 31 of heads t / 32 + 8 i.
    {
        const int p = lane;
        float sn = 0.f, cs = 1.f;
        if (A.rotate) sincosf(static_cast<float>(sq.pos) * A.inv_freq[p], &sn, &cs);
        const float2* Q = reinterpret_cast<const float2*>(A.q + static_cast<size_t>(s) * BNH * BHD);
#pragma unroll
        for (int i = 0; i < BNH / 8; ++i) {
            const int h = warp + 8 * i;
            const float2 x = Q[h * (BHD / 2) + p];
            float y0 = x.x, y1 = x.y;
            if (A.rotate) {
                y0 = x.x * cs - x.y * sn;
                y1 = x.x * sn + x.y * cs;
            }
            *reinterpret_cast<uint32_t*>(&S.q[h * BHD + 2 * p]) = pack_bf16(y0 * 0.125f, y1 * 0.125f);
        }
        // The chunk holding row pos appends bf16(rotated k) and bf16(v)
        // (ops.cpp:1370-1371) before its tiles are read.
        size_t row = 0;
        if (has_new && bf_row<PAGED>(A, sq, sq.pos, row)) {
            if (tid < BROW / 2) {   // k pairs: head tid / 32, pair tid & 31 (= lane)
                const float2 x = reinterpret_cast<const float2*>(A.k + static_cast<size_t>(s) * BROW)[tid];
                float y0 = x.x, y1 = x.y;
                if (A.rotate) {
                    y0 = x.x * cs - x.y * sn;
                    y1 = x.x * sn + x.y * cs;
                }
                reinterpret_cast<uint32_t*>(kc + row)[tid] = pack_bf16(y0, y1);
            } else {
                const int t2 = tid - BROW / 2;
                const float2 x = reinterpret_cast<const float2*>(A.v + static_cast<size_t>(s) * BROW)[t2];
                reinterpret_cast<uint32_t*>(vc + row)[t2] = pack_bf16(x.x, x.y);
            }
            __threadfence();
        }
    }
    __syncthreads();

    // Tile t of the chunk into stage t % BSTAGES: 64 rows x 32 chunks of K
    // and of V, 16 pieces per thread; rows past the chunk are zero-filled.
    const int n_tiles = (nrows + BTILE - 1) / BTILE;
    // (A tile's 64 rows lie in one page: chunks start at multiples of 64 and
    // pages hold a power-of-two multiple of 64 rows.)
    auto issue = [&](int t) {
        const int st = t % BSTAGES;
        const uint32_t kb = smem_u32(S.k[st]), vb = smem_u32(S.v[st]);
        size_t tb = 0;
        const bool tok = bf_row<PAGED>(A, sq, r0 + t * BTILE, tb);
#pragma unroll
        for (int j = 0; j < (BTILE * 32) / BTHREADS; ++j) {
            const int e = tid + j * BTHREADS;
            const int r = e >> 5, ch = e & 31;
            const bool ok = tok && t * BTILE + r < nrows;
            const size_t src = ok ? tb + static_cast<size_t>(r) * BROW + ch * 8 : 0;
            cp16(kb + tile_off(r, ch), kc + src, ok);
            cp16(vb + tile_off(r, ch), vc + src, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
#pragma unroll
    for (int t = 0; t < BSTAGES - 1; ++t) {
        if (t < n_tiles) issue(t);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }

    // A fragments of Q_g (rows = the 8 query heads of KV head g, rows 8-15
    // zero): a0 = (row gid, dims 2 tg + 16 ks ..), a2 = (row gid, + 8).
    const int g = warp & 3, half = warp >> 2;
    const int gid = lane >> 2, tg = lane & 3;
    uint32_t qa0[4], qa2[4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
        const uint16_t* qr = &S.q[(8 * g + gid) * BHD + 16 * ks + 2 * tg];
        qa0[ks] = *reinterpret_cast<const uint32_t*>(qr);
        qa2[ks] = *reinterpret_cast<const uint32_t*>(qr + 8);
    }
    float m = -INFINITY, l = 0.f;     // log2 domain, row gid
    float o[8][4];                    // dims 8 nt + 2 tg (+1): o[nt][0], o[nt][1] (rows 8-15 unused)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    // ldmatrix lane roles: matrix mi = lane / 8, row i = lane % 8
    const int mi = lane >> 3, li = lane & 7;

    for (int t = 0; t < n_tiles; ++t) {
        // the stage of tile t + 2 was released by the barrier ending tile t - 1
        if (t + BSTAGES - 1 < n_tiles) issue(t + BSTAGES - 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group %0;" ::"n"(BSTAGES - 1) : "memory");   // tile t landed
        __syncthreads();
        const int st = t % BSTAGES;
        const uint32_t kbase = smem_u32(S.k[st]), vbase = smem_u32(S.v[st]);
        const int kk0 = 32 * half;   // this warp's keys in the tile
        // S = Q_g K^T for 32 keys: 4 n-tiles of 8 keys
        float sf[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) sf[nt][0] = sf[nt][1] = sf[nt][2] = sf[nt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
            for (int kb = 0; kb < 2; ++kb) {
                uint32_t b0a, b1a, b0b, b1b;
                ldsm_x4(kbase + tile_off(kk0 + 16 * kb + li + 8 * (mi >> 1), 8 * g + 2 * ks + (mi & 1)), b0a, b1a,
                        b0b, b1b);
                mma16816(sf[2 * kb], qa0[ks], qa2[ks], b0a, b1a);
                mma16816(sf[2 * kb + 1], qa0[ks], qa2[ks], b0b, b1b);
            }
        }
        // online softmax of row gid (log2 domain); keys past the chunk masked
        const int key0 = t * BTILE + kk0 + 2 * tg;
        float mt = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const bool ok = key0 + 8 * nt + e < nrows;
                sf[nt][e] = ok ? sf[nt][e] * kLog2e : -INFINITY;
                mt = fmaxf(mt, sf[nt][e]);
            }
        }
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
        const float mn = fmaxf(m, mt);
        const float f = (m == -INFINITY) ? 0.f : ex2f(m - mn);
        m = mn;
        uint32_t pa[4];   // bf16 pairs: n-tile nt's two keys of row gid
        float lsum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            const float p0 = (sf[nt][0] == -INFINITY) ? 0.f : bf16_round(ex2f(sf[nt][0] - mn));
            const float p1 = (sf[nt][1] == -INFINITY) ? 0.f : bf16_round(ex2f(sf[nt][1] - mn));
            lsum += p0 + p1;
            pa[nt] = pack_bf16(p0, p1);
        }
        l = fmaf(l, f, lsum);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            o[nt][0] *= f;
            o[nt][1] *= f;
        }
        // O += P V: k-steps of 16 keys (n-tiles 2 ks2, 2 ks2 + 1 of S), dims in pairs of n-tiles
#pragma unroll
        for (int ks2 = 0; ks2 < 2; ++ks2) {
#pragma unroll
            for (int dp = 0; dp < 4; ++dp) {
                uint32_t b0a, b1a, b0b, b1b;
                ldsm_x4_t(vbase + tile_off(kk0 + 16 * ks2 + li + 8 * (mi & 1), 8 * g + 2 * dp + (mi >> 1)), b0a,
                          b1a, b0b, b1b);
                mma16816(o[2 * dp], pa[2 * ks2], pa[2 * ks2 + 1], b0a, b1a);
                mma16816(o[2 * dp + 1], pa[2 * ks2], pa[2 * ks2 + 1], b0b, b1b);
            }
        }
        __syncthreads();   // the stage is refilled at the next tile
    }
    asm volatile("cp.async.wait_all;" ::: "memory");

    // row sums over the four lanes of a row, then the key halves folded
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (half == 1) {
        float* fr = S.fold[g][lane];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            fr[2 * nt] = o[nt][0];
            fr[2 * nt + 1] = o[nt][1];
        }
        fr[16] = m;
        fr[17] = l;
    }
    __syncthreads();
    if (half == 0) {
        const float* fr = S.fold[g][lane];
        const float m1 = fr[16], l1 = fr[17];
        const float mt = fmaxf(m, m1);   // the first half always has a key: finite
        const float f0 = ex2f(m - mt), f1 = (m1 == -INFINITY) ? 0.f : ex2f(m1 - mt);
        const float lt = l * f0 + l1 * f1;
        const float inv = 1.0f / lt;
        const int h = 8 * g + gid;
        float* dst;
        if (n_chunks == 1) {
            dst = A.out + (static_cast<size_t>(s) * BNH + h) * BHD;
        } else {
            const size_t rec = (static_cast<size_t>(s) * A.max_chunks + c) * BNH + h;
            dst = A.parts + rec * BHD;
            if (tg == 0) A.lses[rec] = (mt + log2f(lt)) * kLn2;   // natural log-sum-exp of the chunk
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
            *reinterpret_cast<float2*>(dst + 8 * nt + 2 * tg) =
                make_float2((o[nt][0] * f0 + fr[2 * nt] * f1) * inv, (o[nt][1] * f0 + fr[2 * nt + 1] * f1) * inv);
    }
}

// Sequences of more than one chunk: out = sum_c w_c o_c, w_c = exp(lse_c -
// LSE), LSE = log sum_c exp(lse_c), in chunk order.  Thread t: head t / 8,
// dims 8 (t % 8) ...
template <bool PAGED>
__global__ void __launch_bounds__(256) merge_bf16_kernel(const __grid_constant__ BfArgs A) {
    asm volatile("griddepcontrol.wait;" ::: "memory");   // the decode's partials
    const int s = blockIdx.x;
    const BfSeqView<PAGED> sq = bf_seq<PAGED>(A, s);
    const int L = sq.pos + 1;
    const int n_chunks = (L + A.chunk - 1) / A.chunk;
    if (n_chunks <= 1 || !sq.ok || n_chunks > A.max_chunks) return;   // reported by the decode
    const int h = threadIdx.x >> 3, d0 = 8 * (threadIdx.x & 7);
    const size_t base = static_cast<size_t>(s) * A.max_chunks * BNH + h;
    float mx = -INFINITY;
    for (int c = 0; c < n_chunks; ++c) mx = fmaxf(mx, A.lses[base + static_cast<size_t>(c) * BNH]);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float wsum = 0.f;
    for (int c = 0; c < n_chunks; ++c) {
        const size_t rec = base + static_cast<size_t>(c) * BNH;
        const float w = expf(A.lses[rec] - mx);
        wsum += w;
        const float4* src = reinterpret_cast<const float4*>(A.parts + rec * BHD + d0);
        const float4 a = src[0], b = src[1];
        acc[0] = fmaf(a.x, w, acc[0]);
        acc[1] = fmaf(a.y, w, acc[1]);
        acc[2] = fmaf(a.z, w, acc[2]);
        acc[3] = fmaf(a.w, w, acc[3]);
        acc[4] = fmaf(b.x, w, acc[4]);
        acc[5] = fmaf(b.y, w, acc[5]);
        acc[6] = fmaf(b.z, w, acc[6]);
        acc[7] = fmaf(b.w, w, acc[7]);
    }
    const float inv = 1.0f / wsum;
    float4* dst = reinterpret_cast<float4*>(A.out + (static_cast<size_t>(s) * BNH + h) * BHD + d0);
    dst[0] = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
    dst[1] = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
}

}  // namespace

size_t decode_bf16_workspace_bytes(int n_seqs, int max_rows) {
    const int chunk = bf16_chunk_rows(n_seqs, max_rows);
    const size_t chunks = static_cast<size_t>((max_rows + chunk - 1) / chunk);
    return static_cast<size_t>(n_seqs) * chunks * BNH * (BHD + 1) * sizeof(float);
}

cudaError_t launch_decode_bf16(const BfArgs& a, cudaStream_t stream) {
    static PerDeviceOnce once;
    cudaError_t e = once.run([&](int) {
        cudaError_t r = cudaFuncSetAttribute(decode_bf16_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(BfSmem)));
        if (r != cudaSuccess) return r;
        return cudaFuncSetAttribute(decode_bf16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(sizeof(BfSmem)));
    });
    if (e != cudaSuccess) return e;
    // both launches are programmatic dependents of the kernel before them
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.max_chunks, a.n_seqs);
    cfg.blockDim = dim3(BTHREADS);
    cfg.dynamicSmemBytes = sizeof(BfSmem);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = a.pseqs ? cudaLaunchKernelEx(&cfg, decode_bf16_kernel<true>, a)
                : cudaLaunchKernelEx(&cfg, decode_bf16_kernel<false>, a);
    if (e != cudaSuccess || a.max_chunks <= 1) return e;
    cfg.gridDim = dim3(a.n_seqs);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    return a.pseqs ? cudaLaunchKernelEx(&cfg, merge_bf16_kernel<true>, a)
                   : cudaLaunchKernelEx(&cfg, merge_bf16_kernel<false>, a);
}

}  // namespace tle
