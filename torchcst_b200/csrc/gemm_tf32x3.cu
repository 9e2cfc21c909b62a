// C = A B^T on Blackwell tensor cores (tcgen05.mma, TMEM accumulator) with
// float32 accuracy from a three-product split:
//     C ~= A_hi B_hi + A_hi B_lo + A_lo B_hi,
// in one of two element formats, both with 11-bit significands:
//   TF32: X_hi = rn_tf32(X), X_lo = rn_tf32(X - X_hi)           (kind::tf32)
//   F16:  X_hi = rn_f16(s X), X_lo = rn_f16(s X - X_hi), with a per-tensor
//         power-of-two s that puts max |s X| in [2^14, 2^15)     (kind::f16)
// The F16 products run at twice the TF32 rate on half the operand bytes; the
// epilogue multiplies by 1 / (s_A s_B), which is exact. Splits are produced
// upstream (tcst_split_tf32, tcst_split_f16).
//
// One CTA computes one 128 x BN output tile of one split-K slice:
//   warp 0       TMA producer: 2-D tiled bulk tensor loads of A_hi, A_lo,
//                B_hi, B_lo per stage (swizzled), completing on the stage's
//                "full" mbarrier;
//   warp 1       TMEM allocator and MMA issuer: 3 x (BK / KSTEP) tcgen05.mma
//                per stage into one fp32 accumulator of BN TMEM columns; a
//                tcgen05.commit frees the stage, a final one signals the epilogue;
//   warps 2..5   epilogue: tcgen05.ld 32 columns at a time, each 32 x 32
//                block transposed through shared memory (the stage buffers
//                are free by then) into whole-row-segment fp32 stores.
// K-major operands are staged as swizzled rows of BK elements; MN-major
// operands as strips of 128 bytes of MN by BK k-rows (TF32: 128-byte swizzle
// with 32-byte units, the MN-major tf32 layout; F16: 128-byte swizzle, with
// 64-byte K-major rows and 4 stages). Every mbarrier wait is bounded: on
// expiry the kernel raises TCST_STATUS_TIMEOUT in the status word and unwinds
// without touching TMEM again except to free it.

#include <cuda.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace tcst {
namespace gemm {

constexpr int BM = 128;
constexpr int THREADS = 192;
constexpr unsigned WAIT_LIMIT = 1u << 22; // a few seconds of try_wait polling

// Staging formats. ESIZE bytes per element; a stage holds BK elements of K;
// one MMA consumes KSTEP elements of K (32 bytes). K-major operands are staged
// as rows of K_ROW = BK * ESIZE bytes (the swizzle span); MN-major operands as
// strips of MN_ROW bytes of MN by BK k-rows. Shared-memory descriptor layout
// types: 2 = 128-byte swizzle, 1 = 128-byte swizzle with 32-byte units (the
// MN-major tf32 layout), 4 = 64-byte swizzle; SBO is the distance between
// 8-row (4-row for type 1) swizzle groups.
struct TF32 {
    static constexpr int ESIZE = 4, BK = 32, KSTEP = 8, K_ROW = 128, MN_ROW = 128, STAGES = 2;
    static constexpr unsigned AB_FORMAT = 2; // instruction-descriptor A/B format
    static constexpr unsigned K_LAYOUT = 2, K_SBO = 1024;
    static constexpr unsigned MN_LAYOUT = 1, MN_SBO = 512;
};
// F16, 64 elements of K per stage: 2 stages of 96 KB (MN-major operands).
struct F16Wide {
    static constexpr int ESIZE = 2, BK = 64, KSTEP = 16, K_ROW = 128, MN_ROW = 128, STAGES = 2;
    static constexpr unsigned AB_FORMAT = 0;
    static constexpr unsigned K_LAYOUT = 2, K_SBO = 1024;
    static constexpr unsigned MN_LAYOUT = 2, MN_SBO = 1024;
};
// F16, 32 elements of K per stage: 4 stages of 48 KB, so three fills are in
// flight while one stage is consumed (the fill latency of a 96 KB stage is
// about one stage's MMA time, which left the tensor pipe waiting with 2
// stages). K-major rows are 64 bytes (64-byte swizzle); MN-major strips stay
// 128 bytes wide. Used when both operands are K-major.
struct F16 {
    static constexpr int ESIZE = 2, BK = 32, KSTEP = 16, K_ROW = 64, MN_ROW = 128, STAGES = 4;
    static constexpr unsigned AB_FORMAT = 0;
    static constexpr unsigned K_LAYOUT = 4, K_SBO = 512;
    static constexpr unsigned MN_LAYOUT = 2, MN_SBO = 1024;
};

template <class P, int BN, int STAGES> struct Layout {
    static constexpr int A_BYTES = BM * P::BK * P::ESIZE;
    static constexpr int B_BYTES = BN * P::BK * P::ESIZE;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
    static constexpr int SMEM_BYTES = BAR_OFFSET + 256 + 1024; // + barriers + alignment slack
};

__device__ __forceinline__ unsigned smem_u32(const void *p) {
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(unsigned bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(unsigned bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: false when the limit expired (the caller unwinds).
__device__ __forceinline__ bool mbar_wait(unsigned bar, unsigned parity) {
    for (unsigned i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ void tma_load_2d(unsigned dst, const CUtensorMap *map, unsigned bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// UMMA shared-memory matrix descriptor with sm_100 version bits (layout types
// as listed with the staging formats above).
__device__ __forceinline__ uint64_t smem_desc(unsigned addr, unsigned lbo, unsigned sbo,
                                              unsigned layout) {
    uint64_t d = 0;
    d |= uint64_t((addr >> 4) & 0x3FFF);
    d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
    d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
    d |= uint64_t(1) << 46; // descriptor version for tcgen05
    d |= uint64_t(layout & 7) << 61;
    return d;
}

template <class P>
__device__ __forceinline__ void mma(unsigned tmem_d, uint64_t a, uint64_t b, unsigned idesc,
                                    unsigned accumulate) {
    if constexpr (P::ESIZE == 4) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
    }
}

__device__ __forceinline__ void mma_commit(unsigned bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// Staged operand geometry. K-major: rows of K_ROW bytes (BK elements),
// swizzled over 8-row groups SBO apart; a k-step is 32 bytes along the row.
// MN-major: strips of MN_ROW bytes of MN (STRIP_ELEMS elements) by BK k-rows
// (BK * MN_ROW bytes, strip stride = LBO); swizzle groups of k-rows are SBO
// apart; a k-step is KSTEP rows.
template <class P, bool MN> struct OperandGeom {
    static constexpr unsigned STRIP = P::BK * unsigned(P::MN_ROW);
    static constexpr int STRIP_ELEMS = P::MN_ROW / P::ESIZE;
    static __device__ __forceinline__ unsigned kstep(int kk) {
        return MN ? kk * unsigned(P::KSTEP) * unsigned(P::MN_ROW) : kk * 32u;
    }
    static __device__ __forceinline__ unsigned lbo() { return MN ? STRIP : 16u; }
    static __device__ __forceinline__ unsigned sbo() { return MN ? P::MN_SBO : P::K_SBO; }
    static __device__ __forceinline__ unsigned layout() {
        return MN ? P::MN_LAYOUT : P::K_LAYOUT;
    }
    static __device__ __forceinline__ uint64_t desc(unsigned addr) {
        return smem_desc(addr, lbo(), sbo(), layout());
    }
};

// Optional MSE epilogue (Y = X W^T of a training step): instead of Y the
// kernel writes dY = (Y - T) * scale, one double sum of (Y - T)^2 per
// epilogue warp into partial[cta * 4 + warp quarter], and max |dY| into amax
// (non-negative floats order like their bit patterns).
struct MseEpilogue {
    const float *target; // nullptr: plain GEMM
    long long ldt;
    float scale;
    double *partial;
    float *amax;
};

template <class P, int BN, int STAGES, bool A_MN, bool B_MN, bool MSE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_x3_kernel(const __grid_constant__ CUtensorMap map_a_hi,
                   const __grid_constant__ CUtensorMap map_a_lo,
                   const __grid_constant__ CUtensorMap map_b_hi,
                   const __grid_constant__ CUtensorMap map_b_lo, int M, int N, int K,
                   int k_per_split, float *__restrict__ C, long long ldc, long long split_stride,
                   const float *__restrict__ scale_a, const float *__restrict__ scale_b,
                   unsigned *__restrict__ status, MseEpilogue mse) {
    using L = Layout<P, BN, STAGES>;
    constexpr int BK = P::BK;
    using GA = OperandGeom<P, A_MN>;
    using GB = OperandGeom<P, B_MN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const unsigned smem_base = smem_u32(smem);
    const unsigned bar_base = smem_base + L::BAR_OFFSET;
    // barriers: full[s] at 8s, empty[s] at 8(STAGES+s), acc at 16*STAGES
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
    const unsigned acc_bar = bar_base + 16u * STAGES;
    volatile unsigned *tmem_slot =
        reinterpret_cast<volatile unsigned *>(smem + L::BAR_OFFSET + 16 * STAGES + 8);
    volatile unsigned *abort_flag = tmem_slot + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tile_n = blockIdx.x, tile_m = blockIdx.y, split = blockIdx.z;
    const int k_begin = split * k_per_split;
    const int k_end = min(K, k_begin + k_per_split);
    const int num_kb = k_end > k_begin ? (k_end - k_begin + BK - 1) / BK : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(acc_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        unsigned slot = smem_u32(const_cast<unsigned *>(tmem_slot));
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
                     "r"(BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (warp == 0 && lane == 0) {
        // Descriptor fetches overlap the previous kernel's tail.
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_a_hi) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_a_lo) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_b_hi) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_b_lo) : "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem_base = *tmem_slot;
    pdl_wait(); // operands and C come from earlier kernels; the setup above does not

    if (warp == 0) {
        if (lane == 0) {
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % STAGES;
                const unsigned phase = (kb / STAGES) & 1;
                if (!mbar_wait(empty_bar(s), phase ^ 1)) {
                    atomicOr(status, TCST_STATUS_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                if (*abort_flag) break;
                const unsigned st = smem_base + s * L::STAGE_BYTES;
                const unsigned a_hi = st, a_lo = st + L::A_BYTES;
                const unsigned b_hi = a_lo + L::A_BYTES, b_lo = b_hi + L::B_BYTES;
                const int k0 = k_begin + kb * BK;
                mbar_expect_tx(full_bar(s), L::STAGE_BYTES);
                if (!A_MN) {
                    tma_load_2d(a_hi, &map_a_hi, full_bar(s), k0, tile_m * BM);
                    tma_load_2d(a_lo, &map_a_lo, full_bar(s), k0, tile_m * BM);
                } else {
#pragma unroll
                    for (int j = 0; j < BM / GA::STRIP_ELEMS; ++j) {
                        const int m0 = tile_m * BM + GA::STRIP_ELEMS * j;
                        tma_load_2d(a_hi + j * GA::STRIP, &map_a_hi, full_bar(s), m0, k0);
                        tma_load_2d(a_lo + j * GA::STRIP, &map_a_lo, full_bar(s), m0, k0);
                    }
                }
                if (!B_MN) {
                    tma_load_2d(b_hi, &map_b_hi, full_bar(s), k0, tile_n * BN);
                    tma_load_2d(b_lo, &map_b_lo, full_bar(s), k0, tile_n * BN);
                } else {
#pragma unroll
                    for (int j = 0; j < BN / GB::STRIP_ELEMS; ++j) {
                        const int n0 = tile_n * BN + GB::STRIP_ELEMS * j;
                        tma_load_2d(b_hi + j * GB::STRIP, &map_b_hi, full_bar(s), n0, k0);
                        tma_load_2d(b_lo + j * GB::STRIP, &map_b_lo, full_bar(s), n0, k0);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // Instruction descriptor: f32 accumulate, A/B format, majors, N>>3, M>>4.
            const unsigned idesc = (1u << 4) | (P::AB_FORMAT << 7) | (P::AB_FORMAT << 10) |
                                   (unsigned(A_MN) << 15) | (unsigned(B_MN) << 16) |
                                   (unsigned(BN >> 3) << 17) | (unsigned(BM >> 4) << 24);
            int issued = 0;
            for (int kb = 0; kb < num_kb; ++kb) {
                const int s = kb % STAGES;
                const unsigned phase = (kb / STAGES) & 1;
                if (!mbar_wait(full_bar(s), phase)) {
                    atomicOr(status, TCST_STATUS_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const unsigned st = smem_base + s * L::STAGE_BYTES;
                const unsigned a_hi = st, a_lo = st + L::A_BYTES;
                const unsigned b_hi = a_lo + L::A_BYTES, b_lo = b_hi + L::B_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / P::KSTEP; ++kk) {
                    const unsigned ao = GA::kstep(kk);
                    const unsigned bo = GB::kstep(kk);
                    const uint64_t dah = GA::desc(a_hi + ao);
                    const uint64_t dal = GA::desc(a_lo + ao);
                    const uint64_t dbh = GB::desc(b_hi + bo);
                    const uint64_t dbl = GB::desc(b_lo + bo);
                    mma<P>(tmem_base, dah, dbh, idesc, issued ? 1u : 0u);
                    mma<P>(tmem_base, dah, dbl, idesc, 1u);
                    mma<P>(tmem_base, dal, dbh, idesc, 1u);
                    issued = 1;
                }
                mma_commit(empty_bar(s));
            }
            mma_commit(acc_bar);
        }
    } else {
        // Epilogue warps 2..5 own TMEM lane quarters (warp % 4): 32 rows each.
        // With the MSE epilogue a warp moves each 32 x 32 block through shared
        // memory (the stage buffers are free once the accumulator is ready),
        // so target loads and dY stores are whole 128-byte row segments.
        const int quarter = warp & 3;
        const int row_base = tile_m * BM + quarter * 32;
        float *out = C + (long long)split * split_stride;
        if (MSE && row_base + lane < M) {
            // The target tile is read only after the accumulator is ready:
            // bring its lines into L2 while the MMAs run.
            const float *tr = mse.target + (long long)(row_base + lane) * mse.ldt + tile_n * BN;
            const int ncol = min(BN, N - tile_n * BN);
            for (int c = 0; c < ncol; c += 32) {
                asm volatile("prefetch.global.L2 [%0];" ::"l"(tr + c));
                asm volatile("prefetch.global.L2 [%0];" ::"l"(tr + min(c + 31, ncol - 1)));
            }
        }
        bool ready = true;
        if (num_kb > 0) {
            ready = mbar_wait(acc_bar, 0);
            if (!ready) atomicOr(status, TCST_STATUS_TIMEOUT);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        }
        double loss = 0.0;
        float vmax = 0.f;
        if (ready && !*abort_flag) {
            // 1 / (s_A s_B): a power of two, so the product is exact.
            const float inv = (scale_a && scale_b) ? 1.0f / (*scale_a * *scale_b) : 1.0f;
            const bool vec = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
            float *blk = reinterpret_cast<float *>(smem) + quarter * (32 * 36);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                unsigned r[32];
                if (num_kb > 0) {
                    const unsigned taddr = tmem_base + (unsigned(quarter * 32) << 16) + unsigned(c0);
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
                          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]),
                          "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                        : "r"(taddr));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) r[j] = 0u;
                }
                const int col0 = tile_n * BN + c0;
                if (!MSE && !(vec && col0 + 32 <= N)) {
                    // Ragged or unaligned output: each lane stores its row.
                    const int row = row_base + lane;
                    if (row < M) {
                        float *dst = out + (long long)row * ldc + col0;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < N) dst[j] = __uint_as_float(r[j]) * inv;
                    }
                    continue;
                }
                // The 32 x 32 block goes through shared memory, lane = row on
                // the way in (float4 writes, pitch 36: each 8-lane phase hits
                // 32 distinct banks), so that the global accesses are whole
                // 128-byte row segments.
                {
                    float4 *b4 = reinterpret_cast<float4 *>(blk + lane * 36);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        b4[j] = make_float4(__uint_as_float(r[4 * j]) * inv,
                                            __uint_as_float(r[4 * j + 1]) * inv,
                                            __uint_as_float(r[4 * j + 2]) * inv,
                                            __uint_as_float(r[4 * j + 3]) * inv);
                }
                __syncwarp();
                if (!MSE) {
                    // Eight lanes per row, four rows per store instruction.
                    const int sub = lane >> 3, c4 = 4 * (lane & 7);
#pragma unroll
                    for (int rr = 0; rr < 32; rr += 4) {
                        const int row = row_base + rr + sub;
                        if (row < M)
                            *reinterpret_cast<float4 *>(out + (long long)row * ldc + col0 + c4) =
                                *reinterpret_cast<const float4 *>(blk + (rr + sub) * 36 + c4);
                    }
                    __syncwarp();
                    continue;
                }
                // MSE: lane = column on the way out.
                const int col = tile_n * BN + c0 + lane;
                const bool col_ok = col < N;
                {
                    // dY = (Y - T) * scale in place of Y; sum (Y - T)^2 in double.
                    float t[32];
#pragma unroll
                    for (int rr = 0; rr < 32; ++rr) {
                        const int row = row_base + rr;
                        t[rr] = row < M && col_ok ? mse.target[(long long)row * mse.ldt + col] : 0.f;
                    }
#pragma unroll
                    for (int rr = 0; rr < 32; ++rr) {
                        const int row = row_base + rr;
                        if (row < M && col_ok) {
                            const float d = blk[rr * 36 + lane] - t[rr];
                            loss += double(d) * double(d);
                            const float g = d * mse.scale;
                            vmax = fmaxf(vmax, fabsf(g));
                            out[(long long)row * ldc + col] = g;
                        }
                    }
                }
                __syncwarp();
            }
        }
        if (MSE) {
            // One loss partial per epilogue warp (fixed xor tree), one max
            // atomic per warp.
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                loss += __shfl_xor_sync(0xffffffffu, loss, o);
                vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
            }
            if (lane == 0) {
                mse.partial[(blockIdx.y * (long long)gridDim.x + blockIdx.x) * 4 + quarter] = loss;
                if (mse.amax && vmax > 0.f)
                    atomicMax(reinterpret_cast<unsigned *>(mse.amax), __float_as_uint(vmax));
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(BN));
    }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps and launch.
// ---------------------------------------------------------------------------

using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                              const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                              const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
    static EncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFn>(p);
    });
    return fn;
}

// 2-D map over a row-major [outer][inner] array with leading dimension ld
// (elements), box {one staged row of inner, box_outer}, zero fill outside the
// array; swizzle over that row (MN-major TF32: 128 bytes with 32-byte units).
template <class P>
static int make_map(CUtensorMap *map, const void *base, long long inner, long long outer,
                    long long ld, int box_outer, bool mn_major) {
    EncodeFn fn = encode_fn();
    if (!fn) {
        tcst_set_error("cuTensorMapEncodeTiled is unavailable from the driver");
        return TCST_ERR_CUDA;
    }
    cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(outer)};
    cuuint64_t strides[1] = {cuuint64_t(ld) * P::ESIZE};
    const int row = mn_major ? P::MN_ROW : P::K_ROW;
    cuuint32_t box[2] = {cuuint32_t(row / P::ESIZE), cuuint32_t(box_outer)};
    cuuint32_t estr[2] = {1u, 1u};
    const CUtensorMapDataType dt =
        P::ESIZE == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUtensorMapSwizzle sw = row == 64                     ? CU_TENSOR_MAP_SWIZZLE_64B
                                  : (mn_major && P::ESIZE == 4) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                                : CU_TENSOR_MAP_SWIZZLE_128B;
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        tcst_set_error("cuTensorMapEncodeTiled failed (%d) for inner=%lld outer=%lld ld=%lld",
                       int(r), inner, outer, ld);
        return TCST_ERR_CUDA;
    }
    return TCST_OK;
}

// C = 0 for an empty contraction (K == 0): no operand is read.
__global__ void zero_fill_kernel(float *__restrict__ C, long long M, long long N, long long ldc,
                                 long long split_stride, int splits) {
    pdl_wait();
    long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long per = M * N;
    if (idx >= per * splits) return;
    long long s = idx / per, r = (idx % per) / N, c = idx % N;
    C[s * split_stride + r * ldc + c] = 0.0f;
}

template <class P, int BN, int STAGES, bool A_MN, bool B_MN, bool MSE = false>
static int launch(int M, int N, int K, const CUtensorMap *maps, int kps, int splits, float *C,
                  long long ldc, long long sstride, const float *sa, const float *sb,
                  unsigned *status, cudaStream_t stream, const MseEpilogue &mse) {
    using L = Layout<P, BN, STAGES>;
    auto kern = gemm_x3_kernel<P, BN, STAGES, A_MN, B_MN, MSE>;
    static bool configured = false;
    if (!configured) {
        TCST_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::SMEM_BYTES));
        configured = true;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, splits);
    TCST_CUDA(launch_pdl(kern, dim3(grid), dim3(THREADS), L::SMEM_BYTES, stream, maps[0], maps[1], maps[2], maps[3], M, N, K, kps,
                                                   C, ldc, sstride, sa, sb, status, mse));
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

// Shared host path of both formats.
template <class P>
static int gemm_x3(const char *name, int64_t M, int64_t N, int64_t K, const void *a_hi_dev,
                   const void *a_lo_dev, int64_t lda, int32_t a_mn_major, const void *b_hi_dev,
                   const void *b_lo_dev, int64_t ldb, int32_t b_mn_major, float *c_dev,
                   int64_t ldc, int32_t split_k, int64_t split_stride, const float *sa,
                   const float *sb, uint32_t *status_dev, void *stream,
                   const MseEpilogue &mse = MseEpilogue{}) {
    if (M < 0 || N < 0 || K < 0 || split_k < 1 || !status_dev || M > INT32_MAX ||
        N > INT32_MAX || K > INT32_MAX) {
        tcst_set_error("%s: invalid sizes", name);
        return TCST_ERR_ARGUMENT;
    }
    if (M == 0 || N == 0) return TCST_OK;
    if (!c_dev || ldc < N || (split_k > 1 && split_stride < M * ldc)) {
        tcst_set_error("%s: NULL output or invalid output layout", name);
        return TCST_ERR_ARGUMENT;
    }
    if (K == 0) {
        long long total = M * N * split_k;
        TCST_CUDA(launch_pdl(zero_fill_kernel, dim3(unsigned((total + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, 
            c_dev, M, N, ldc, split_stride, split_k));
        TCST_CUDA(cudaGetLastError());
        return TCST_OK;
    }
    if (!a_hi_dev || !a_lo_dev || !b_hi_dev || !b_lo_dev) {
        tcst_set_error("%s: NULL operand", name);
        return TCST_ERR_ARGUMENT;
    }
    const long long a_inner = a_mn_major ? M : K, a_outer = a_mn_major ? K : M;
    const long long b_inner = b_mn_major ? N : K, b_outer = b_mn_major ? K : N;
    const int align = 16 / P::ESIZE; // elements per 16 bytes
    if (lda < a_inner || ldb < b_inner || lda % align || ldb % align ||
        ((reinterpret_cast<uintptr_t>(a_hi_dev) | reinterpret_cast<uintptr_t>(a_lo_dev) |
          reinterpret_cast<uintptr_t>(b_hi_dev) | reinterpret_cast<uintptr_t>(b_lo_dev)) & 15)) {
        tcst_set_error("%s: operands need 16-byte aligned bases and rows", name);
        return TCST_ERR_ARGUMENT;
    }
    constexpr int BN = 256;
    constexpr int STAGES = P::STAGES;
    constexpr int BK = P::BK;
    CUtensorMap maps[4];
    int rc;
    const int a_box = a_mn_major ? BK : BM;
    const int b_box = b_mn_major ? BK : BN;
    if ((rc = make_map<P>(&maps[0], a_hi_dev, a_inner, a_outer, lda, a_box, a_mn_major)) ||
        (rc = make_map<P>(&maps[1], a_lo_dev, a_inner, a_outer, lda, a_box, a_mn_major)) ||
        (rc = make_map<P>(&maps[2], b_hi_dev, b_inner, b_outer, ldb, b_box, b_mn_major)) ||
        (rc = make_map<P>(&maps[3], b_lo_dev, b_inner, b_outer, ldb, b_box, b_mn_major)))
        return rc;
    // Split K into whole BK blocks.
    long long kb_total = (K + BK - 1) / BK;
    long long kb_per = (kb_total + split_k - 1) / split_k;
    int kps = int(kb_per * BK);
    cudaStream_t st = (cudaStream_t)stream;
    unsigned *status = status_dev;
    if (!a_mn_major && !b_mn_major) {
        if (mse.target)
            return launch<P, BN, STAGES, false, false, true>(int(M), int(N), int(K), maps, kps,
                                                             split_k, c_dev, ldc, split_stride,
                                                             sa, sb, status, st, mse);
        return launch<P, BN, STAGES, false, false>(int(M), int(N), int(K), maps, kps, split_k,
                                                   c_dev, ldc, split_stride, sa, sb, status, st,
                                                   mse);
    }
    if (!a_mn_major && b_mn_major)
        return launch<P, BN, STAGES, false, true>(int(M), int(N), int(K), maps, kps, split_k,
                                                  c_dev, ldc, split_stride, sa, sb, status, st,
                                                  mse);
    if (a_mn_major && !b_mn_major)
        return launch<P, BN, STAGES, true, false>(int(M), int(N), int(K), maps, kps, split_k,
                                                  c_dev, ldc, split_stride, sa, sb, status, st,
                                                  mse);
    return launch<P, BN, STAGES, true, true>(int(M), int(N), int(K), maps, kps, split_k, c_dev,
                                             ldc, split_stride, sa, sb, status, st, mse);
}

} // namespace gemm
} // namespace tcst

using namespace tcst;
using namespace tcst::gemm;

extern "C" int tcst_gemm_tf32x3(int64_t M, int64_t N, int64_t K, const float *a_hi_dev,
                                const float *a_lo_dev, int64_t lda, int32_t a_mn_major,
                                const float *b_hi_dev, const float *b_lo_dev, int64_t ldb,
                                int32_t b_mn_major, float *c_dev, int64_t ldc, int32_t split_k,
                                int64_t split_stride, uint32_t *status_dev, void *stream) {
    return gemm_x3<TF32>("tcst_gemm_tf32x3", M, N, K, a_hi_dev, a_lo_dev, lda, a_mn_major,
                         b_hi_dev, b_lo_dev, ldb, b_mn_major, c_dev, ldc, split_k, split_stride,
                         nullptr, nullptr, status_dev, stream);
}

extern "C" int tcst_gemm_f16x3(int64_t M, int64_t N, int64_t K, const void *a_hi_dev,
                               const void *a_lo_dev, int64_t lda, int32_t a_mn_major,
                               const float *a_scale_dev, const void *b_hi_dev,
                               const void *b_lo_dev, int64_t ldb, int32_t b_mn_major,
                               const float *b_scale_dev, float *c_dev, int64_t ldc,
                               int32_t split_k, int64_t split_stride, uint32_t *status_dev,
                               void *stream) {
    if (M > 0 && N > 0 && K > 0 && (!a_scale_dev || !b_scale_dev)) {
        tcst_set_error("tcst_gemm_f16x3: NULL operand scale");
        return TCST_ERR_ARGUMENT;
    }
    // Four 48 KB stages measured faster when both operands are K-major (Y =
    // X W^T: 29.5 vs 31.6 us at 4096 x 1024 x 1024); with an MN-major operand
    // two 96 KB stages are as fast or faster.
    if (!a_mn_major && !b_mn_major)
        return gemm_x3<F16>("tcst_gemm_f16x3", M, N, K, a_hi_dev, a_lo_dev, lda, a_mn_major,
                            b_hi_dev, b_lo_dev, ldb, b_mn_major, c_dev, ldc, split_k,
                            split_stride, a_scale_dev, b_scale_dev, status_dev, stream);
    return gemm_x3<F16Wide>("tcst_gemm_f16x3", M, N, K, a_hi_dev, a_lo_dev, lda, a_mn_major,
                        b_hi_dev, b_lo_dev, ldb, b_mn_major, c_dev, ldc, split_k, split_stride,
                        a_scale_dev, b_scale_dev, status_dev, stream);
}

extern "C" int tcst_gemm_f16x3_mse(int64_t M, int64_t N, int64_t K, const void *a_hi_dev,
                                   const void *a_lo_dev, int64_t lda, const float *a_scale_dev,
                                   const void *b_hi_dev, const void *b_lo_dev, int64_t ldb,
                                   const float *b_scale_dev, const float *target_dev,
                                   int64_t ld_target, float scale, float *dy_dev, int64_t ld_dy,
                                   double *loss_partial_dev, int32_t *partials,
                                   float *amax_dev, uint32_t *status_dev, void *stream) {
    const int64_t tiles = ((N + 255) / 256) * ((M + BM - 1) / BM);
    if (partials) *partials = int32_t(tiles * 4);
    if (M < 0 || N < 0 || K < 1 || !target_dev || ld_target < N || !loss_partial_dev ||
        !a_scale_dev || !b_scale_dev) {
        tcst_set_error("tcst_gemm_f16x3_mse: invalid arguments (K must be positive)");
        return TCST_ERR_ARGUMENT;
    }
    const MseEpilogue mse{target_dev, ld_target, scale, loss_partial_dev, amax_dev};
    return gemm_x3<F16>("tcst_gemm_f16x3_mse", M, N, K, a_hi_dev, a_lo_dev, lda, 0, b_hi_dev,
                        b_lo_dev, ldb, 0, dy_dev, ld_dy, 1, 0, a_scale_dev, b_scale_dev,
                        status_dev, stream, mse);
}
