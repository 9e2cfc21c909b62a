// C = A B^T on Blackwell tensor cores (tcgen05.mma kind::tf32, TMEM accumulator)
// with float32 accuracy from the three-product TF32 split:
//     C ~= A_hi B_hi + A_hi B_lo + A_lo B_hi,
// where X_hi = rn_tf32(X) and X_lo = rn_tf32(X - X_hi) are produced upstream.
//
// One CTA computes one 128 x BN output tile of one split-K slice:
//   warp 0       TMA producer: four 2-D tiled bulk tensor loads per stage
//                (A_hi, A_lo, B_hi, B_lo; 128-byte swizzle), completing on the
//                stage's "full" mbarrier;
//   warp 1       TMEM allocator and MMA issuer: 3 x (BK / 8) tcgen05.mma per
//                stage into one fp32 accumulator of BN TMEM columns; a
//                tcgen05.commit frees the stage, a final one signals the epilogue;
//   warps 2..5   epilogue: tcgen05.ld 32 columns at a time, fp32 stores.
// K-major operands are staged as [rows][32] float rows (128-byte swizzle,
// 16-byte units); MN-major operands as 32-element strips of [32 k][32] (4 KiB
// each, 128-byte swizzle with 32-byte units, the MN-major tf32 layout). Every mbarrier wait is bounded: on expiry the kernel raises
// TCST_STATUS_TIMEOUT in the status word and unwinds without touching TMEM
// again except to free it.

#include <cuda.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace tcst {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 32; // fp32 elements per 128-byte swizzle row
constexpr int THREADS = 192;
constexpr unsigned WAIT_LIMIT = 1u << 22; // a few seconds of try_wait polling

template <int BN, int STAGES> struct Layout {
    static constexpr int A_BYTES = BM * BK * 4;
    static constexpr int B_BYTES = BN * BK * 4;
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

// UMMA shared-memory matrix descriptor with sm_100 version bits. Layout type 2
// is the 128-byte swizzle with 16-byte units (K-major operands); layout type 1
// is the 128-byte swizzle with 32-byte units, the only MN-major layout for
// 32-bit (tf32) operands.
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

__device__ __forceinline__ void mma_tf32(unsigned tmem_d, uint64_t a, uint64_t b, unsigned idesc,
                                         unsigned accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(unsigned bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// Staged operand geometry. K-major: [rows][32] fp32 rows of 128 bytes, 16-byte
// swizzle units over 8-row (1024-byte) groups. MN-major: 32-element MN strips of
// [32 k][32] (4 KiB, strip stride = LBO), 32-byte swizzle units over 4-row
// (512-byte) groups (= SBO).
template <bool MN> struct OperandGeom {
    // Byte offset of k-step kk (8 fp32 of K) inside one staged operand.
    static __device__ __forceinline__ unsigned kstep(int kk) { return MN ? kk * 1024u : kk * 32u; }
    static __device__ __forceinline__ unsigned lbo() { return MN ? 4096u : 16u; }
    static __device__ __forceinline__ unsigned sbo() { return MN ? 512u : 1024u; }
    static __device__ __forceinline__ unsigned layout() { return MN ? 1u : 2u; }
    static __device__ __forceinline__ uint64_t desc(unsigned addr) {
        return smem_desc(addr, lbo(), sbo(), layout());
    }
};

template <int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap map_a_hi,
                       const __grid_constant__ CUtensorMap map_a_lo,
                       const __grid_constant__ CUtensorMap map_b_hi,
                       const __grid_constant__ CUtensorMap map_b_lo, int M, int N, int K,
                       int k_per_split, float *__restrict__ C, long long ldc,
                       long long split_stride, unsigned *__restrict__ status) {
    using L = Layout<BN, STAGES>;
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
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem_base = *tmem_slot;

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
                    for (int j = 0; j < BM / 32; ++j) {
                        tma_load_2d(a_hi + j * 4096, &map_a_hi, full_bar(s), tile_m * BM + 32 * j, k0);
                        tma_load_2d(a_lo + j * 4096, &map_a_lo, full_bar(s), tile_m * BM + 32 * j, k0);
                    }
                }
                if (!B_MN) {
                    tma_load_2d(b_hi, &map_b_hi, full_bar(s), k0, tile_n * BN);
                    tma_load_2d(b_lo, &map_b_lo, full_bar(s), k0, tile_n * BN);
                } else {
#pragma unroll
                    for (int j = 0; j < BN / 32; ++j) {
                        tma_load_2d(b_hi + j * 4096, &map_b_hi, full_bar(s), tile_n * BN + 32 * j, k0);
                        tma_load_2d(b_lo + j * 4096, &map_b_lo, full_bar(s), tile_n * BN + 32 * j, k0);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // Instruction descriptor: f32 accumulate, tf32 A/B, majors, N>>3, M>>4.
            const unsigned idesc = (1u << 4) | (2u << 7) | (2u << 10) | (unsigned(A_MN) << 15) |
                                   (unsigned(B_MN) << 16) | (unsigned(BN >> 3) << 17) |
                                   (unsigned(BM >> 4) << 24);
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
                for (int kk = 0; kk < BK / 8; ++kk) {
                    const unsigned ao = OperandGeom<A_MN>::kstep(kk);
                    const unsigned bo = OperandGeom<B_MN>::kstep(kk);
                    const uint64_t dah = OperandGeom<A_MN>::desc(a_hi + ao);
                    const uint64_t dal = OperandGeom<A_MN>::desc(a_lo + ao);
                    const uint64_t dbh = OperandGeom<B_MN>::desc(b_hi + bo);
                    const uint64_t dbl = OperandGeom<B_MN>::desc(b_lo + bo);
                    mma_tf32(tmem_base, dah, dbh, idesc, issued ? 1u : 0u);
                    mma_tf32(tmem_base, dah, dbl, idesc, 1u);
                    mma_tf32(tmem_base, dal, dbh, idesc, 1u);
                    issued = 1;
                }
                mma_commit(empty_bar(s));
            }
            mma_commit(acc_bar);
        }
    } else {
        // Epilogue warps 2..5 own TMEM lane quarters (warp % 4).
        const int quarter = warp & 3;
        const int row = tile_m * BM + quarter * 32 + lane;
        float *out = C + (long long)split * split_stride;
        bool ready = true;
        if (num_kb > 0) {
            ready = mbar_wait(acc_bar, 0);
            if (!ready) atomicOr(status, TCST_STATUS_TIMEOUT);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        }
        if (ready && !*abort_flag) {
            const bool vec = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
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
                if (row < M) {
                    const int col0 = tile_n * BN + c0;
                    float *dst = out + (long long)row * ldc + col0;
                    if (vec && col0 + 32 <= N) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4 *>(dst + j) =
                                make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                            __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < N) dst[j] = __uint_as_float(r[j]);
                    }
                }
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

// 2-D fp32 map over a row-major [outer][inner] array with leading dimension ld,
// box {32, box_outer}, zero fill outside the array; 128-byte swizzle with 16-byte
// units for K-major operands, 32-byte units for MN-major ones.
static int make_map(CUtensorMap *map, const float *base, long long inner, long long outer,
                    long long ld, int box_outer, bool mn_major) {
    EncodeFn fn = encode_fn();
    if (!fn) {
        tcst_set_error("cuTensorMapEncodeTiled is unavailable from the driver");
        return TCST_ERR_CUDA;
    }
    cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(outer)};
    cuuint64_t strides[1] = {cuuint64_t(ld) * 4};
    cuuint32_t box[2] = {32u, cuuint32_t(box_outer)};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        tcst_set_error("cuTensorMapEncodeTiled failed (%d) for inner=%lld outer=%lld ld=%lld",
                       int(r), inner, outer, ld);
        return TCST_ERR_CUDA;
    }
    return TCST_OK;
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
static int launch(int M, int N, int K, const CUtensorMap *maps, int kps, int splits, float *C,
                  long long ldc, long long sstride, unsigned *status, cudaStream_t stream) {
    using L = Layout<BN, STAGES>;
    auto kern = gemm_tf32x3_kernel<BN, STAGES, A_MN, B_MN>;
    static bool configured = false;
    if (!configured) {
        TCST_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::SMEM_BYTES));
        configured = true;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, splits);
    kern<<<grid, THREADS, L::SMEM_BYTES, stream>>>(maps[0], maps[1], maps[2], maps[3], M, N, K, kps,
                                                   C, ldc, sstride, status);
    TCST_CUDA(cudaGetLastError());
    return TCST_OK;
}

// C = 0 for an empty contraction (K == 0): no operand is read.
__global__ void zero_fill_kernel(float *__restrict__ C, long long M, long long N, long long ldc,
                                 long long split_stride, int splits) {
    long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long per = M * N;
    if (idx >= per * splits) return;
    long long s = idx / per, r = (idx % per) / N, c = idx % N;
    C[s * split_stride + r * ldc + c] = 0.0f;
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
    if (M < 0 || N < 0 || K < 0 || split_k < 1 || !status_dev || M > INT32_MAX ||
        N > INT32_MAX || K > INT32_MAX) {
        tcst_set_error("tcst_gemm_tf32x3: invalid sizes");
        return TCST_ERR_ARGUMENT;
    }
    if (M == 0 || N == 0) return TCST_OK;
    if (!c_dev || ldc < N || (split_k > 1 && split_stride < M * ldc)) {
        tcst_set_error("tcst_gemm_tf32x3: NULL output or invalid output layout");
        return TCST_ERR_ARGUMENT;
    }
    if (K == 0) {
        long long total = M * N * split_k;
        zero_fill_kernel<<<unsigned((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
            c_dev, M, N, ldc, split_stride, split_k);
        TCST_CUDA(cudaGetLastError());
        return TCST_OK;
    }
    if (!a_hi_dev || !a_lo_dev || !b_hi_dev || !b_lo_dev) {
        tcst_set_error("tcst_gemm_tf32x3: NULL operand");
        return TCST_ERR_ARGUMENT;
    }
    const long long a_inner = a_mn_major ? M : K, a_outer = a_mn_major ? K : M;
    const long long b_inner = b_mn_major ? N : K, b_outer = b_mn_major ? K : N;
    if (lda < a_inner || ldb < b_inner || lda % 4 || ldb % 4 ||
        ((reinterpret_cast<uintptr_t>(a_hi_dev) | reinterpret_cast<uintptr_t>(a_lo_dev) |
          reinterpret_cast<uintptr_t>(b_hi_dev) | reinterpret_cast<uintptr_t>(b_lo_dev)) & 15)) {
        tcst_set_error("tcst_gemm_tf32x3: operands need 16-byte aligned bases and ld %% 4 == 0");
        return TCST_ERR_ARGUMENT;
    }
    constexpr int BN = 256;
    constexpr int STAGES = 2;
    CUtensorMap maps[4];
    int rc;
    const int a_box = a_mn_major ? BK : BM;
    const int b_box = b_mn_major ? BK : BN;
    if ((rc = make_map(&maps[0], a_hi_dev, a_inner, a_outer, lda, a_box, a_mn_major)) ||
        (rc = make_map(&maps[1], a_lo_dev, a_inner, a_outer, lda, a_box, a_mn_major)) ||
        (rc = make_map(&maps[2], b_hi_dev, b_inner, b_outer, ldb, b_box, b_mn_major)) ||
        (rc = make_map(&maps[3], b_lo_dev, b_inner, b_outer, ldb, b_box, b_mn_major)))
        return rc;
    // Split K into whole BK blocks.
    long long kb_total = (K + BK - 1) / BK;
    long long kb_per = (kb_total + split_k - 1) / split_k;
    int kps = int(kb_per * BK);
    cudaStream_t st = (cudaStream_t)stream;
    unsigned *status = status_dev;
    if (!a_mn_major && !b_mn_major)
        return launch<BN, STAGES, false, false>(int(M), int(N), int(K), maps, kps, split_k, c_dev, ldc,
                                                split_stride, status, st);
    if (!a_mn_major && b_mn_major)
        return launch<BN, STAGES, false, true>(int(M), int(N), int(K), maps, kps, split_k, c_dev, ldc,
                                               split_stride, status, st);
    if (a_mn_major && !b_mn_major)
        return launch<BN, STAGES, true, false>(int(M), int(N), int(K), maps, kps, split_k, c_dev, ldc,
                                               split_stride, status, st);
    return launch<BN, STAGES, true, true>(int(M), int(N), int(K), maps, kps, split_k, c_dev, ldc,
                                          split_stride, status, st);
}
