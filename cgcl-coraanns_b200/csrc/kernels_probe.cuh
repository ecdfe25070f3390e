// Coarse probing on the tensor cores: approximate squared distances of every (query,
// centroid) pair, approx = |q'|^2 + |c|^2 - 2 <q', c>, with <q', c> from tcgen05 TF32 MMAs.
//
// Reference: the query x centroid SGEMM and distance epilogue of hybrid.cu:436-470 (cuBLAS +
// a RAFT select_k); here the GEMM is one persistent warp-specialised sm_100a kernel and the
// selection stays exact through guarded_select_kernel, which recomputes every centroid in
// the error band in fp64 (so the probe lists are bit-identical to the reference's exact
// selection whatever the GEMM's rounding).
//
// Error bound used by the guard (kApproxEpsTF32): TF32 keeps 10 mantissa bits of each input
// (truncation, relative error <= 2^-10), so every product has relative error <= 2^-9 + 2^-20;
// fp32 accumulation over D <= 1024 terms adds <= D * 2^-23 <= 2^-13 of sum |q_i c_i|. Hence
// |d<q',c>| <= 2^-8.9 |q'||c| and |d approx| <= 2^-7.9 |q'||c| <= 2^-9.9 (|q'| + c_max)^2;
// the guard uses eps = 2^-9, about twice that.
//
// Kernel layout (one CTA per SM, 192 threads):
//   warp 0     TMA producer: 128 x 32 query tile + 256 x 32 centroid tile per stage
//              (K-major, 128-byte swizzle), kStages stages in flight;
//   warp 1     allocates 512 TMEM columns (two 128 x 256 fp32 accumulators) and issues the
//              MMAs (M 128, N 256, K 8) from one lane; tcgen05.commit frees stages and
//              publishes accumulators;
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time, apply the norms, stage the
//              128 x 32 block in shared memory (128-byte swizzle) and TMA-store it; with
//              chunk_min, also each row's minimum over every 32-column chunk
//              (chunk_min[q * chunk_stride(nlist) + c / 32], +inf past nlist), which lets
//              the selection read only the chunks that can hold a probe.
// Every wait is bounded (kDevWaitTimeout on expiry) and the CTA always drains its copies and
// MMAs and frees its TMEM before it exits.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace cora {

constexpr int kPgBM = 128, kPgBN = 256, kPgBK = 32;  // tile rows, cols; K floats per stage
constexpr int kPgStages = 4;
constexpr int kPgThreads = 192;
constexpr uint32_t kPgStageA = kPgBM * kPgBK * 4;  // 16 KB
constexpr uint32_t kPgStageB = kPgBN * kPgBK * 4;  // 32 KB
constexpr uint32_t kPgOutBuf = kPgBM * 32 * 4;     // 16 KB, two of them
constexpr uint32_t kPgTmemCols = 512;
constexpr double kApproxEpsTF32 = 1.0 / 512.0;

__host__ __device__ constexpr size_t probe_gemm_smem() {
    return 1024 /* alignment slack */ + (size_t)kPgStages * (kPgStageA + kPgStageB) +
           2 * kPgOutBuf + 256 /* barriers + TMEM slot */;
}

// ---- PTX wrappers (sm_100a) -------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *smem_src, int x,
                                             int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(smem_src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group_read1() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
                 : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, both K-major, kind::tf32.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}
// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (one lane = one thread).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with 128-byte swizzle:
// rows of 128 bytes, 8-row atoms 1024 bytes apart (stride byte offset), leading byte offset
// 16 (unused by swizzled K-major layouts), descriptor version 1, layout type 2
// (SWIZZLE_128B). The tile base must be 1024-byte aligned (base offset 0).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void *p) {
    const uint64_t addr = smem_u32(p);
    return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
// Instruction descriptor: fp32 accumulator, A and B tf32, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__global__ void __launch_bounds__(kPgThreads, 1) probe_gemm_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_c,
    const __grid_constant__ CUtensorMap tm_out, const float *__restrict__ qnorm2,
    const float *__restrict__ cnorm2, int nq, int nlist, int D, float *__restrict__ chunk_min,
    int qfast, int *err) {
    extern __shared__ unsigned char pg_smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(pg_smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *sA = smem;
    unsigned char *sB = smem + kPgStages * kPgStageA;
    unsigned char *sOut = sB + kPgStages * kPgStageB;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sOut + 2 * kPgOutBuf);
    uint64_t *full = bars, *empty = bars + kPgStages;
    uint64_t *tfull = bars + 2 * kPgStages, *tempty = tfull + 2, *mma_done = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    // Tile order. qfast (large centroid matrices): query-block-fastest, so the CTAs of a
    // wave share one or two centroid blocks (read from DRAM once, then from L2) while the
    // query matrix stays in L2; centroid-block-fastest, every wave streamed the whole
    // centroid matrix again (3.75 GB of DRAM reads for 131 MB of operands at config 4).
    // Otherwise centroid-block-fastest: the centroids stay in L2 anyway and a wave writes
    // whole output rows (config 2: 0.060 against 0.072 ms).
    const int ntn = (nlist + kPgBN - 1) / kPgBN;
    const int ntm = (nq + kPgBM - 1) / kPgBM;
    const int tiles = ntm * ntn;
    const int KC = D / kPgBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPgStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull + b, 1);
            mbar_init(tempty + b, 4);  // one arrival per epilogue warp
        }
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kPgTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t s = 0, ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int m0 = (qfast ? t % ntm : t / ntn) * kPgBM, n0 = (qfast ? t / ntm : t % ntn) * kPgBN;
                for (int kc = 0; kc < KC; ++kc) {
                    if (!(ok = mbar_wait_bounded(empty + s, ph ^ 1, err))) break;
                    mbar_arrive_expect_tx(full + s, kPgStageA + kPgStageB);
                    tma_load_2d(sA + s * kPgStageA, &tm_q, kc * kPgBK, m0, full + s);
                    tma_load_2d(sB + s * kPgStageB, &tm_c, kc * kPgBK, n0, full + s);
                    if (++s == kPgStages) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            // drain: the last load issued into each stage has landed before the CTA exits
            for (int i = 0; i < kPgStages; ++i) {
                if (s == 0) ph ^= 1;
                s = (s + kPgStages - 1) % kPgStages;
                mbar_wait_bounded(full + s, ph, err);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(kPgBM, kPgBN);
            uint32_t s = 0, ph = 0, acc = 0, aph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                if (!(ok = mbar_wait_bounded(tempty + acc, aph ^ 1, err))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + acc * kPgBN;
                for (int kc = 0; kc < KC; ++kc) {
                    if (!(ok = mbar_wait_bounded(full + s, ph, err))) break;
                    tc_fence_after();
                    const uint64_t a0 = smem_desc_sw128(sA + s * kPgStageA);
                    const uint64_t b0 = smem_desc_sw128(sB + s * kPgStageB);
#pragma unroll
                    for (int kk = 0; kk < kPgBK / 8; ++kk)  // K = 8 tf32 = 32 bytes per MMA
                        mma_tf32(d_tmem, a0 + 2 * kk, b0 + 2 * kk, idesc, (kc | kk) != 0);
                    mma_commit(empty + s);
                    if (++s == kPgStages) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                mma_commit(tfull + acc);
                if (++acc == 2) {
                    acc = 0;
                    aph ^= 1;
                }
            }
            mma_commit(mma_done);  // every MMA issued has finished before TMEM is freed
            mbar_wait_bounded(mma_done, 0, err);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int et = threadIdx.x - 64;             // 0..127
        const int quarter = warp & 3;                // TMEM lanes this warp may read
        const int row = quarter * 32 + lane;         // tile row = TMEM lane
        uint32_t acc = 0, aph = 0, obuf = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            const int m0 = (qfast ? t % ntm : t / ntn) * kPgBM, n0 = (qfast ? t / ntm : t % ntn) * kPgBN;
            ok = ok && mbar_wait_bounded(tfull + acc, aph, err);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
            // every epilogue thread takes part in the barriers below even after a timeout
            tc_fence_after();
            const int q = m0 + row;
            const float qn = (ok && q < nq) ? __ldg(qnorm2 + q) : 0.0f;
            float cm8[kPgBN / 32];  // this row's minima of the tile's eight 32-column chunks
#pragma unroll
            for (int j = 0; j < kPgBN / 32; ++j) {
                float v[32];
                if (ok) {
                    tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + acc * kPgBN + j * 32, v);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0.0f;
                }
                const int c0 = n0 + j * 32;
                if (et == 0) bulk_wait_group_read1();  // this buffer's previous store is read
                named_barrier_sync(1, 128);
                unsigned char *ob = sOut + obuf * kPgOutBuf + row * 128;
                // cnorm2 is zero-padded to a multiple of 256: whole-chunk vector loads are safe
                const float4 *cn4 = reinterpret_cast<const float4 *>(cnorm2 + c0);
                float cmin = __int_as_float(0x7f800000);  // min over the chunk's columns
                const bool full = c0 + 32 <= nlist;
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    const float4 cn = __ldg(cn4 + ch);
                    float4 o;
                    o.x = __fsub_rn(__fadd_rn(qn, cn.x), __fmul_rn(2.0f, v[ch * 4 + 0]));
                    o.y = __fsub_rn(__fadd_rn(qn, cn.y), __fmul_rn(2.0f, v[ch * 4 + 1]));
                    o.z = __fsub_rn(__fadd_rn(qn, cn.z), __fmul_rn(2.0f, v[ch * 4 + 2]));
                    o.w = __fsub_rn(__fadd_rn(qn, cn.w), __fmul_rn(2.0f, v[ch * 4 + 3]));
                    if (full) {
                        cmin = fminf(cmin, fminf(fminf(o.x, o.y), fminf(o.z, o.w)));
                    } else {  // the row's last, partial chunk: padded columns stay out
                        const int c = c0 + ch * 4;
                        if (c < nlist) cmin = fminf(cmin, o.x);
                        if (c + 1 < nlist) cmin = fminf(cmin, o.y);
                        if (c + 2 < nlist) cmin = fminf(cmin, o.z);
                        if (c + 3 < nlist) cmin = fminf(cmin, o.w);
                    }
                    *reinterpret_cast<float4 *>(ob + ((ch ^ (row & 7)) << 4)) = o;
                }
                cm8[j] = cmin;  // +inf for chunks past nlist
                fence_proxy_async_smem();
                named_barrier_sync(1, 128);
                if (et == 0 && ok) {
                    tma_store_2d(&tm_out, sOut + obuf * kPgOutBuf, c0, m0);
                    bulk_commit_group();
                }
                obuf ^= 1;
            }
            if (chunk_min && ok && q < nq) {  // one full 32-byte sector per row and tile
                float4 *dst = reinterpret_cast<float4 *>(
                    chunk_min + (size_t)q * chunk_stride(nlist) + n0 / 32);
                dst[0] = make_float4(cm8[0], cm8[1], cm8[2], cm8[3]);
                dst[1] = make_float4(cm8[4], cm8[5], cm8[6], cm8[7]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty + acc);
            if (++acc == 2) {
                acc = 0;
                aph ^= 1;
            }
        }
        if (et == 0) bulk_wait_group_all();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kPgTmemCols);
}

}  // namespace cora
