// gemv.cu -- the reference's weight path on the device (sm_100a):
// read_tensor_f32 (GGUF F32 / F16 / Q4_0 / Q8_0 -> f32) and matmul_f64
// (y = x . W over a weight tensor), crates/compiler/src/gguf_compiler.rs:
// 351-470 and :1239-1255 in SugarFreeDoNoSo/bml.
//
// Layout.  The reference keeps a tensor's values in file order and reads
// W[i][j] at flat index i*n_out + j, where (n_in, n_out) = (dims[0],
// dims[1]) -- so row i of W is n_out consecutive values, and a quantized
// block (32 consecutive values) covers 32 consecutive columns of one row
// when n_out is a multiple of 32.
//
// Dequantisation follows the reference bit for bit: f16 scales widen
// exactly, Q4_0 byte i of a block holds elements 2i (low nibble) and 2i+1
// (high nibble), value (q - 8) * scale; Q8_0 value q * scale; blocks that do
// not fit in the data are zero.
//
// GEMV (HBM-bound: every weight byte is read once, ~2 flops per element).
// The quantized tensor is read as stored -- 0.5625 bytes per value for
// Q4_0 instead of the 4 bytes of the reference's dequantised f32 pool.  A
// CTA owns 256 columns (8 blocks of 32) and a range of rows; thread t takes
// block t % 8 and rows r = t / 8 (mod 32) of the range, keeping 32 f32 sums.
// Each term is x[i] * scale (f32, once per block and row) times (q - 8) or
// q, the small integer made exact with the 2^23 magic-number trick (no
// int-to-float conversion unit in the loop).  The 32 row phases are summed
// in f64 in a fixed order, and the row ranges (when a tensor needs several
// CTAs per column range to fill the GPU) go to a workspace in f64 and are
// summed in a fixed order by a second kernel, so results do not vary between
// runs; against the reference's f64 sums they differ by f32 rounding of the
// terms and partial sums (about 1e-7 of sum |x_i W_ij|).
#include "gemv.cuh"

namespace bml {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kColBlocks = 8;                  // 32-column blocks per CTA
constexpr int kCols = kColBlocks * 32;         // columns per CTA
constexpr int kRowPhases = kGemvThreads / kColBlocks;  // 32
constexpr uint64_t kMaxRanges = 160;                  // row ranges of one GEMV
constexpr uint32_t kReduceLoads = (kMaxRanges + 7) / 8;  // ranges a reduce thread adds: 20

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Exact small integers as floats: 2^23 + u has u in its low mantissa bits,
// so (2^23 + u) - (2^23 + off) = u - off exactly (u < 2^23), in one FADD.
__device__ __forceinline__ float magic_u(uint32_t u, float off) {
    return __uint_as_float(0x4B000000u | u) - (8388608.0f + off);
}

// ------------------------------------------------------------ dequant
// One thread per 32-value block.
template <int QT>
__global__ void dequant_q_kernel(const uint8_t *__restrict__ data, uint64_t n_blocks_ok, uint64_t n_elems,
                                 float *__restrict__ out) {
    const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t n_blocks = (n_elems + 31) / 32;
    if (b >= n_blocks) return;
    float v[32];
    if (b < n_blocks_ok) {
        constexpr uint32_t BB = QT == kGgufQ4_0 ? 18u : 34u;
        const uint16_t *blk = reinterpret_cast<const uint16_t *>(data + b * BB);  // 2-byte aligned
        const float scale = f16_bits_to_f32(blk[0]);
        if (QT == kGgufQ4_0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t two = blk[1 + i];  // bytes 2i, 2i+1 of the 16 nibble bytes
#pragma unroll
                for (int k = 0; k < 4; ++k) v[4 * i + k] = magic_u((two >> (4 * k)) & 15u, 8.0f) * scale;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t two = blk[1 + i];
#pragma unroll
                for (int k = 0; k < 2; ++k) v[2 * i + k] = magic_u(((two >> (8 * k)) & 255u) ^ 128u, 128.0f) * scale;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
    }
    const uint64_t base = b * 32;
    if (base + 32 <= n_elems) {
        float4 *o = reinterpret_cast<float4 *>(out + base);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
        for (int i = 0; i < 32 && base + i < n_elems; ++i) out[base + i] = v[i];
    }
}

__global__ void dequant_f16_kernel(const uint16_t *__restrict__ data, uint64_t n, float *__restrict__ out) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = f16_bits_to_f32(data[i]);
}

// ------------------------------------------------------------ GEMV
// The 32 values of W in row i, columns [32*cb, 32*cb + 32), times xs.
template <int QT>
struct Block32 {
    __device__ __forceinline__ static void fma(const uint8_t *__restrict__ w, uint64_t row, uint64_t n_out,
                                               uint64_t cb, uint64_t n_blocks_ok, double x, float acc[32]) {
        const uint64_t b = row * (n_out / 32) + cb;
        if (b >= n_blocks_ok) return;  // past the data: zeros
        constexpr uint32_t BB = QT == kGgufQ4_0 ? 18u : 34u;
        const uint16_t *blk = reinterpret_cast<const uint16_t *>(w + b * BB);
        const float xs = (float)x * f16_bits_to_f32(__ldg(blk));
        if (QT == kGgufQ4_0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t two = __ldg(blk + 1 + i);
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[4 * i + k] = fmaf(xs, magic_u((two >> (4 * k)) & 15u, 8.0f), acc[4 * i + k]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t two = __ldg(blk + 1 + i);
#pragma unroll
                for (int k = 0; k < 2; ++k)
                    acc[2 * i + k] = fmaf(xs, magic_u(((two >> (8 * k)) & 255u) ^ 128u, 128.0f), acc[2 * i + k]);
            }
        }
    }
};

template <>
struct Block32<kGgufF32> {
    __device__ __forceinline__ static void fma(const uint8_t *__restrict__ w, uint64_t row, uint64_t n_out,
                                               uint64_t cb, uint64_t n_vals, double x, float acc[32]) {
        const uint64_t e0 = row * n_out + cb * 32;
        if (e0 >= n_vals) return;
        const float xf = (float)x;
        const float *p = reinterpret_cast<const float *>(w) + e0;
        if (e0 + 32 <= n_vals && (n_out % 4) == 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 q = __ldg(reinterpret_cast<const float4 *>(p) + i);
                acc[4 * i] = fmaf(xf, q.x, acc[4 * i]);
                acc[4 * i + 1] = fmaf(xf, q.y, acc[4 * i + 1]);
                acc[4 * i + 2] = fmaf(xf, q.z, acc[4 * i + 2]);
                acc[4 * i + 3] = fmaf(xf, q.w, acc[4 * i + 3]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (e0 + i < n_vals) acc[i] = fmaf(xf, __ldg(p + i), acc[i]);
        }
    }
};

template <>
struct Block32<kGgufF16> {
    __device__ __forceinline__ static void fma(const uint8_t *__restrict__ w, uint64_t row, uint64_t n_out,
                                               uint64_t cb, uint64_t n_vals, double x, float acc[32]) {
        const uint64_t e0 = row * n_out + cb * 32;
        if (e0 >= n_vals) return;
        const float xf = (float)x;
        const uint16_t *p = reinterpret_cast<const uint16_t *>(w) + e0;
        if (e0 + 32 <= n_vals && (n_out % 8) == 0) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 q = __ldg(reinterpret_cast<const uint4 *>(p) + i);
                const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wd[k]));
                    acc[8 * i + 2 * k] = fmaf(xf, f.x, acc[8 * i + 2 * k]);
                    acc[8 * i + 2 * k + 1] = fmaf(xf, f.y, acc[8 * i + 2 * k + 1]);
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (e0 + i < n_vals) acc[i] = fmaf(xf, f16_bits_to_f32(__ldg(p + i)), acc[i]);
        }
    }
};

// grid (column tiles, row ranges); partial[range][n_out] (or y when there
// is one range).
template <int QT>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const uint8_t *__restrict__ w, uint64_t n_ok,
                                                            uint64_t n_out, uint64_t rows, uint64_t rows_per_range,
                                                            const double *__restrict__ x, double *__restrict__ dst) {
    __shared__ float part[kRowPhases][kCols + 1];
    const int tid = threadIdx.x;
    const int cbl = tid % kColBlocks, rp = tid / kColBlocks;
    const uint64_t cb = (uint64_t)blockIdx.x * kColBlocks + cbl;  // global 32-column block
    const uint64_t n_cb = (n_out + 31) / 32;
    const uint64_t r0 = (uint64_t)blockIdx.y * rows_per_range;
    const uint64_t r1 = min(r0 + rows_per_range, rows);
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    if (cb < n_cb) {
#pragma unroll 4
        for (uint64_t r = r0 + rp; r < r1; r += kRowPhases) Block32<QT>::fma(w, r, n_out, cb, n_ok, __ldg(x + r), acc);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) part[rp][cbl * 32 + i] = acc[i];
    __syncthreads();
    // one column per thread: the 32 row phases in order, in f64
    const uint64_t j = (uint64_t)blockIdx.x * kCols + tid;
    if (j < n_out) {
        double s = 0.0;
#pragma unroll 8
        for (int k = 0; k < kRowPhases; ++k) s += (double)part[k][tid];
        dst[(uint64_t)blockIdx.y * n_out + j] = s;
    }
}

// ---- staged GEMV: 1024-column tiles, row segments streamed through a
// cp.async ring in shared memory.  Used when n_out % 256 == 0, W is 16-byte
// aligned and the data holds the whole tensor (rows are then 16-byte
// aligned runs of n_out/32 blocks).  The direct kernel above has each
// thread wait on its own scattered 2-byte loads, one row after another;
// here 256 threads keep three stages of whole row segments (and the x
// values of those rows) in flight.  Thread t owns 32-column block t % 32 of
// the tile and rows t / 32 (mod 8) of each stage.
constexpr int kTileBlocks = 32;
constexpr int kRing = 3;

template <int QT>
struct StagedCfg {
    static constexpr uint32_t BB = QT == kGgufQ4_0 ? 18u : QT == kGgufQ8_0 ? 34u : QT == kGgufF16 ? 64u : 128u;
    static constexpr uint32_t SEG = kTileBlocks * BB;  // bytes of one row of a tile
    static constexpr uint32_t RS_RAW = 18432u / SEG;
    static constexpr uint32_t RS = RS_RAW < 8u ? 8u : (RS_RAW / 8u) * 8u;  // rows per stage
    static constexpr uint32_t XOFF = RS * SEG;        // the stage's RS values of x (f64) follow its rows
    static constexpr uint32_t STAGE = XOFF + RS * 8u;
    static constexpr uint32_t SMEM = kRing * STAGE > 8u * 1056u * 4u ? kRing * STAGE : 8u * 1056u * 4u;
};

__device__ __forceinline__ void cp8(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// acc[i] += x * (values 2i, 2i+1 of the one block at shared address blk),
// in packed f32x2 arithmetic (each lane rounds as fmaf does), for Q8_0, F16
// and F32 (Q4_0 has its own kernel below).  A Q8_0 value becomes a float
// with one byte permute: its byte lane is moved into the low mantissa byte
// of 2^23 (the float then reads 2^23 + q), and one packed add removes the
// offset, exactly.
template <int QT>
__device__ __forceinline__ void block_fma_smem(const uint8_t *blk, float x, float2 acc[16]) {
    if constexpr (QT == kGgufQ8_0) {
        const uint16_t *h = reinterpret_cast<const uint16_t *>(blk);
        const float xs = x * f16_bits_to_f32(h[0]);
        const float2 xs2 = make_float2(xs, xs);
        const float2 off = make_float2(-8388736.0f, -8388736.0f);  // 2^23 + 128
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            // quant bytes 4m..4m+3 (values 4m..4m+3), int8 -> q + 128
            const uint32_t w = __byte_perm(h[1 + 2 * m], h[2 + 2 * m], 0x5410) ^ 0x80808080u;
#pragma unroll
            for (int b = 0; b < 4; b += 2) {
                const float2 q = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440 + b)),
                                             __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441 + b)));
                acc[2 * m + b / 2] = __ffma2_rn(xs2, __fadd2_rn(q, off), acc[2 * m + b / 2]);
            }
        }
    } else if constexpr (QT == kGgufF16) {
        const uint4 *q4 = reinterpret_cast<const uint4 *>(blk);
        const float2 x2 = make_float2(x, x);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 q = q4[i];
            const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int k = 0; k < 4; ++k)
                acc[4 * i + k] = __ffma2_rn(x2, __half22float2(*reinterpret_cast<const __half2 *>(&wd[k])),
                                            acc[4 * i + k]);
        }
    } else {
        const float4 *f4 = reinterpret_cast<const float4 *>(blk);
        const float2 x2 = make_float2(x, x);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 q = f4[i];
            acc[2 * i] = __ffma2_rn(x2, make_float2(q.x, q.y), acc[2 * i]);
            acc[2 * i + 1] = __ffma2_rn(x2, make_float2(q.z, q.w), acc[2 * i + 1]);
        }
    }
}

template <int QT>
__global__ void __launch_bounds__(kGemvThreads, 4) gemv_staged_kernel(const uint8_t *__restrict__ w, uint64_t n_out,
                                                                   uint64_t rows, uint64_t rows_per_range,
                                                                   const double *__restrict__ x,
                                                                   double *__restrict__ dst) {
    using Cf = StagedCfg<QT>;
    extern __shared__ __align__(16) uint8_t sm[];
    const int tid = threadIdx.x;
    const int cbl = tid % kTileBlocks, rp = tid / kTileBlocks;  // 8 row phases
    const uint64_t n_cb = n_out / 32;
    const uint64_t row_bytes = n_cb * Cf::BB;
    const uint64_t cb0 = (uint64_t)blockIdx.x * kTileBlocks;
    // blocks of this tile: a multiple of 8 (n_out % 256 == 0)
    const uint32_t tile_blocks = (uint32_t)(n_cb - cb0 < (uint64_t)kTileBlocks ? n_cb - cb0 : (uint64_t)kTileBlocks);
    const uint32_t seg_chunks = tile_blocks * Cf::BB / 16u;  // <= 256
    // this thread's chunks of a stage: chunk tid, tid + 256, ... as (row,
    // chunk in row), stepped without a division per chunk
    const uint32_t rr0 = (uint32_t)tid / seg_chunks, cc0 = (uint32_t)tid % seg_chunks;
    const uint32_t d_rr = (uint32_t)kGemvThreads / seg_chunks, d_cc = (uint32_t)kGemvThreads % seg_chunks;
    const uint64_t r0 = (uint64_t)blockIdx.y * rows_per_range;
    const uint64_t r1 = min(r0 + rows_per_range, rows);
    const uint32_t n_stages = (uint32_t)((r1 - r0 + Cf::RS - 1) / Cf::RS);
    const uint8_t *tile = w + cb0 * Cf::BB;
    const uint32_t smem0 = (uint32_t)__cvta_generic_to_shared(sm);

    auto stage_rows = [&](uint32_t st) {
        const uint64_t rb = r0 + (uint64_t)st * Cf::RS;
        return (uint32_t)(r1 - rb < (uint64_t)Cf::RS ? r1 - rb : (uint64_t)Cf::RS);
    };
    auto issue = [&](uint32_t st) {  // rows [r0 + st*RS, ...) into ring slot st % kRing
        if (st < n_stages) {
            const uint64_t rb = r0 + (uint64_t)st * Cf::RS;
            const uint32_t nr = stage_rows(st);
            const uint32_t slot = smem0 + (st % kRing) * Cf::STAGE;
            uint32_t rr = rr0, cc = cc0;
            while (rr < nr) {
                cp16(slot + rr * Cf::SEG + cc * 16u, tile + (rb + rr) * row_bytes + cc * 16u);
                rr += d_rr;
                cc += d_cc;
                if (cc >= seg_chunks) {
                    cc -= seg_chunks;
                    ++rr;
                }
            }
            // the stage's x values ride along: no global load in the compute loop
            if ((uint32_t)tid < nr) cp8(slot + Cf::XOFF + tid * 8u, x + rb + tid);
        }
        cp_commit();  // one group per stage, empty past the end
    };

    float2 acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.f, 0.f);
#pragma unroll
    for (int st = 0; st < kRing - 1; ++st) issue(st);
    for (uint32_t st = 0; st < n_stages; ++st) {
        issue(st + kRing - 1);
        cp_wait<kRing - 1>();  // stage st has landed (this thread's copies)
        __syncthreads();       // ... and every thread's
        const uint64_t rb = r0 + (uint64_t)st * Cf::RS;
        const uint32_t nr = stage_rows(st);
        if ((uint32_t)cbl < tile_blocks) {
            const uint8_t *slot = sm + (st % kRing) * Cf::STAGE;
            const double *xst = reinterpret_cast<const double *>(slot + Cf::XOFF);
            constexpr uint32_t kStep = kGemvThreads / kTileBlocks;
            if (nr == Cf::RS) {  // full stage: a fixed trip count, unrolled for independent loads
#pragma unroll
                for (uint32_t k = 0; k < Cf::RS / kStep; ++k) {
                    const uint32_t rr = rp + k * kStep;
                    block_fma_smem<QT>(slot + rr * Cf::SEG + cbl * Cf::BB, (float)xst[rr], acc);
                }
            } else {
                for (uint32_t rr = rp; rr < nr; rr += kStep)
                    block_fma_smem<QT>(slot + rr * Cf::SEG + cbl * Cf::BB, (float)xst[rr], acc);
            }
        }
        __syncthreads();  // the slot is refilled next iteration
    }
    cp_wait<0>();
    __syncthreads();
    // the 8 row phases of each column, summed in f64 in phase order; block
    // cbl's 32 columns sit at word cbl * 33 of phase row rp, so the 32 lanes
    // of a store (32 blocks) land in 32 banks
    float *part = reinterpret_cast<float *>(sm);  // [8][32 * 33]
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        part[rp * 1056 + cbl * 33 + 2 * i] = acc[i].x;
        part[rp * 1056 + cbl * 33 + 2 * i + 1] = acc[i].y;
    }
    __syncthreads();
    for (uint32_t c = tid; c < tile_blocks * 32u; c += kGemvThreads) {
        double sacc = 0.0;
#pragma unroll
        for (int k = 0; k < kGemvThreads / kTileBlocks; ++k) sacc += (double)part[k * 1056 + (c >> 5) * 33 + (c & 31u)];
        dst[(uint64_t)blockIdx.y * n_out + cb0 * 32 + c] = sacc;
    }
}

// ---- staged GEMV for Q4_0: the same tiles, row ranges, row phases and
// order of every sum as gemv_staged_kernel (so the same result bits as the
// generic staged form), at a third of its device time on B200.
//  * A thread owns a PAIR of adjacent blocks of the tile (36 bytes, 4-byte
//    aligned at 36p) and one row phase: 16 pairs x 8 phases = 128 threads,
//    64 f32 sums a thread; nine 4-byte shared loads bring a pair's two
//    scales and 32 quant bytes.  Block 0's quant bytes 0, 1 and 14, 15
//    share words with the scales and are gathered into one word by one byte
//    permute; every other quant word is used as loaded, and which sum slot
//    holds which column is fixed per thread and undone at the end.
//  * A nibble at bits 4k..4k+3 of a word becomes a float with one LOP3
//    (inline: the compiler splits the AND and the OR otherwise):
//    OR-ing in the exponent of 2^(23-4k) makes the mantissa bit 4k weigh 1,
//    so the float reads 2^(23-4k) + q exactly; one packed add of
//    -(2^(23-4k) + 8) leaves q - 8, exactly, for each lane.  The two
//    nibbles of a byte share one packed add and one packed FMA.
//  * Stages of 32 rows, ONE stage ahead (a ring of two): every CTA of the
//    one-wave grid keeps ~18 KB in flight, ~10 MB over the GPU, enough to
//    stream HBM while the data arrive in about the order they are used.
//    Measured on B200 (4096 x 14336): two or three stages ahead, or an L2
//    prefetch of the whole range at the start, put all 33 MB in flight at
//    once and made a CTA's first stage land after ~3.5-5.5 us instead of
//    ~2-3 us (13.8 -> 14.6-16.3 us a launch pair); 16-row stages held too
//    little in flight.  A row is copied by 4 threads, 9 16-byte chunks each
//    at immediate offsets from one address (copy loops with a division per
//    chunk cost ~1.8 us; one bulk copy per 576-byte row, or a 2-D tensor
//    copy per stage, streamed no faster).
//  * The weights of stage 0 may be requested before griddepcontrol.wait, x
//    and everything else after it: launched as a programmatic dependent of
//    the previous kernel (bml_matmul_f64_static), the first weight bytes
//    stream while that kernel ends (~1.1 us of a 4096 x 14336 launch pair
//    measured); launched plainly the wait does nothing.
//  * The phase sums go through shared memory with each pair's 64 columns
//    at a 66-word stride: the 16 lanes of a half-warp's 64-bit store fill
//    all 32 banks.  (An unpadded [8][1024] array made every store a 32-way
//    conflict: 3.2 us of a 18 us launch.)
constexpr int kQ4Threads = 128;
constexpr int kQ4Pairs = kTileBlocks / 2;          // 16
constexpr int kQ4Phases = kQ4Threads / kQ4Pairs;    // 8, as gemv_staged_kernel
constexpr uint32_t kQ4Rows = 32;                    // rows a stage
constexpr uint32_t kQ4Seg = kTileBlocks * 18u;      // 576 bytes of a row in a tile
constexpr uint32_t kQ4XOff = kQ4Rows * kQ4Seg;      // the stage's x values (f64) follow its rows
constexpr uint32_t kQ4Stage = kQ4XOff + kQ4Rows * 8u;
constexpr uint32_t kQ4PartStride = 1056;            // words a phase row: 16 pairs x 66
constexpr uint32_t kQ4Smem = 2 * kQ4Stage > 8 * kQ4PartStride * 4 ? 2 * kQ4Stage : 8 * kQ4PartStride * 4;

// (a & M) | c in one LOP3.  Written as C, the AND and the OR compile to two
// instructions (measured on B200 by instruction-class counters: 17 integer
// instructions per quant word instead of 9), and the integer pipe is what
// limits this kernel.
template <uint32_t M>
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "n"(M), "r"(c));
    return d;
}

// Exponent fields that make mantissa bit 4k weigh 1: 2^23, 2^19, 2^15, 2^11.
struct Q4Magic {
    uint32_t m0 = 0x4B000000u, m1 = 0x49000000u, m2 = 0x47000000u, m3 = 0x45000000u;
};

// acc[0..3] += xs * (q - 8) for the 8 nibbles of quant word w (byte c of w:
// low nibble into acc[c].x, high nibble into acc[c].y).
__device__ __forceinline__ void q4_word(uint32_t w, float2 xs2, float2 *acc, const Q4Magic &mg) {
    const float2 off01 = make_float2(-8388616.0f, -524296.0f);  // -(2^23 + 8), -(2^19 + 8)
    const float2 off23 = make_float2(-32776.0f, -2056.0f);      // -(2^15 + 8), -(2^11 + 8)
    const uint32_t u = w >> 16;
    float2 q;
    q = make_float2(__uint_as_float(and_or<0x000Fu>(w, mg.m0)), __uint_as_float(and_or<0x00F0u>(w, mg.m1)));
    acc[0] = __ffma2_rn(xs2, __fadd2_rn(q, off01), acc[0]);
    q = make_float2(__uint_as_float(and_or<0x0F00u>(w, mg.m2)), __uint_as_float(and_or<0xF000u>(w, mg.m3)));
    acc[1] = __ffma2_rn(xs2, __fadd2_rn(q, off23), acc[1]);
    q = make_float2(__uint_as_float(and_or<0x000Fu>(u, mg.m0)), __uint_as_float(and_or<0x00F0u>(u, mg.m1)));
    acc[2] = __ffma2_rn(xs2, __fadd2_rn(q, off01), acc[2]);
    q = make_float2(__uint_as_float(and_or<0x0F00u>(u, mg.m2)), __uint_as_float(and_or<0xF000u>(u, mg.m3)));
    acc[3] = __ffma2_rn(xs2, __fadd2_rn(q, off23), acc[3]);
}

// Quant byte held by sum slot s (0..15) of a pair's first block: slots 0-3
// hold bytes 0, 1, 14, 15 (the gathered word), slots 4-15 bytes 2-13.  The
// second block's slots 16-31 hold its bytes 0-15 in order.
__device__ __forceinline__ uint32_t q4_slot_byte(uint32_t s) {
    return s >= 16u ? s - 16u : s >= 4u ? s - 2u : (s < 2u ? s : s + 12u);
}

__global__ void __launch_bounds__(kQ4Threads, 4) gemv_q4_kernel(const uint8_t *__restrict__ w, uint64_t n_out,
                                                               uint64_t rows, uint64_t rows_per_range,
                                                               const double *__restrict__ x,
                                                               double *__restrict__ dst) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int tid = threadIdx.x;
    const uint32_t pr = (uint32_t)tid % kQ4Pairs, rp = (uint32_t)tid / kQ4Pairs;
    const uint64_t n_cb = n_out / 32;
    const uint64_t row_bytes = n_cb * 18u;
    const uint64_t cb0 = (uint64_t)blockIdx.x * kTileBlocks;
    const uint32_t tile_blocks = (uint32_t)(n_cb - cb0 < (uint64_t)kTileBlocks ? n_cb - cb0 : (uint64_t)kTileBlocks);
    const uint32_t seg_chunks = tile_blocks * 18u / 16u;  // 36 for a whole tile
    const uint64_t r0 = (uint64_t)blockIdx.y * rows_per_range;
    const uint64_t r1 = min(r0 + rows_per_range, rows);
    const uint32_t n_stages = (uint32_t)((r1 - r0 + kQ4Rows - 1) / kQ4Rows);
    const uint32_t smem0 = (uint32_t)__cvta_generic_to_shared(sm);
    // this thread copies row cr of each stage, chunks cc, cc + 4, ...
    const uint32_t cr = (uint32_t)tid / 4u, cc = (uint32_t)tid % 4u;
    const uint8_t *src0 = w + cb0 * 18u + (uint64_t)cr * row_bytes + cc * 16u;

    auto stage_rows = [&](uint32_t st) {
        const uint64_t rb = r0 + (uint64_t)st * kQ4Rows;
        return (uint32_t)(r1 - rb < (uint64_t)kQ4Rows ? r1 - rb : (uint64_t)kQ4Rows);
    };
    auto issue_w = [&](uint32_t st) {  // the stage's row segments
        if (st >= n_stages) return;
        const uint32_t nr = stage_rows(st);
        if (cr >= nr) return;
        const uint8_t *src = src0 + (r0 + (uint64_t)st * kQ4Rows) * row_bytes;
        const uint32_t dst_s = smem0 + (st & 1u) * kQ4Stage + cr * kQ4Seg + cc * 16u;
        if (seg_chunks == 36u) {
#pragma unroll
            for (uint32_t j = 0; j < 9; ++j) cp16(dst_s + 64u * j, src + 64u * j);
        } else {
            for (uint32_t c = cc; c < seg_chunks; c += 4u) cp16(dst_s + (c - cc) * 16u, src + (c - cc) * 16u);
        }
    };
    auto issue_x = [&](uint32_t st) {  // the stage's x values, then the stage's copy group
        if (st < n_stages && (uint32_t)tid < stage_rows(st))
            cp8(smem0 + (st & 1u) * kQ4Stage + kQ4XOff + tid * 8u, x + r0 + (uint64_t)st * kQ4Rows + tid);
        cp_commit();
    };

    float2 acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = make_float2(0.f, 0.f);
    const Q4Magic mg;
    auto pair_row = [&](const uint8_t *slot, uint32_t rr) {
        const uint32_t *wd = reinterpret_cast<const uint32_t *>(slot + rr * kQ4Seg + pr * 36u);
        uint32_t W[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) W[i] = wd[i];
        const float xf = (float)reinterpret_cast<const double *>(slot + kQ4XOff)[rr];
        const float xs0 = xf * __low2float(*reinterpret_cast<const __half2 *>(&W[0]));
        const float xs1 = xf * __high2float(*reinterpret_cast<const __half2 *>(&W[4]));
        const float2 x0 = make_float2(xs0, xs0), x1 = make_float2(xs1, xs1);
        q4_word(__byte_perm(W[0], W[4], 0x5432), x0, acc + 0, mg);
        q4_word(W[1], x0, acc + 4, mg);
        q4_word(W[2], x0, acc + 8, mg);
        q4_word(W[3], x0, acc + 12, mg);
        q4_word(W[5], x1, acc + 16, mg);
        q4_word(W[6], x1, acc + 20, mg);
        q4_word(W[7], x1, acc + 24, mg);
        q4_word(W[8], x1, acc + 28, mg);
    };

    // Stage 0's weights go out before the wait only when the range has at
    // least 3 stages: with one or two, stage 0 is most of the tensor, and
    // loading it early only competes with the previous kernel's own stream
    // (4096 x 4096, one stage a range: 6.7 us a launch pair without, 8.5
    // with; 4096 x 14336, four stages: 14.0 without, 12.7 with).
    const bool early = n_stages >= 3;
    if (early) issue_w(0);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x (and dst) belong to the previous kernel until here
    if (!early) issue_w(0);
    issue_x(0);
    for (uint32_t st = 0; st < n_stages; ++st) {
        cp_wait<0>();     // stage st has landed (this thread's copies)
        __syncthreads();  // ... and every thread's; the other slot was consumed at st - 1
        issue_w(st + 1);
        issue_x(st + 1);
        const uint32_t nr = stage_rows(st);
        if (pr * 2u < tile_blocks) {
            const uint8_t *slot = sm + (st & 1u) * kQ4Stage;
            if (nr == kQ4Rows) {
#pragma unroll
                for (uint32_t k = 0; k < kQ4Rows / kQ4Phases; ++k) pair_row(slot, rp + k * kQ4Phases);
            } else {
                for (uint32_t rr = rp; rr < nr; rr += kQ4Phases) pair_row(slot, rr);
            }
        }
    }
    cp_wait<0>();
    __syncthreads();
    // the 8 row phases of each column, summed in f64 in phase order; pair
    // pr's 64 columns sit at word pr * 66 of phase row rp
    float *part = reinterpret_cast<float *>(sm);
#pragma unroll
    for (uint32_t s = 0; s < 32; ++s) {
        const uint32_t col = (s >= 16u ? 32u : 0u) + 2u * q4_slot_byte(s);
        *reinterpret_cast<float2 *>(part + rp * kQ4PartStride + pr * 66u + col) = acc[s];
    }
    __syncthreads();
    for (uint32_t c = tid; c < tile_blocks * 32u; c += kQ4Threads) {
        const uint32_t o = (c >> 6) * 66u + (c & 63u);
        double sacc = 0.0;
#pragma unroll
        for (int k = 0; k < kQ4Phases; ++k) sacc += (double)part[k * kQ4PartStride + o];
        dst[(uint64_t)blockIdx.y * n_out + cb0 * 32 + c] = sacc;
    }
}

// y[j] = sum of the row ranges' partials.  A CTA takes 32 columns; warp g
// sums ranges g, g+8, g+16, ... of them in that order, and the 8 group sums
// are added in group order: a fixed association, so results do not vary
// between runs.  A thread's (at most 20) loads are all issued before the
// first add: with each add chained on its load the loop paid one L2 round
// trip per range (the 148-range 14336 x 4096 projection: 17.2 -> 15.0 us a
// launch pair).  Launched as a programmatic dependent of the range kernel:
// its CTAs may start while that kernel ends and wait here for its partials.
__global__ void __launch_bounds__(256) gemv_reduce_kernel(const double *__restrict__ partial, uint32_t n_ranges,
                                                          uint64_t n_out, double *__restrict__ y) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ double grp[8][33];
    const uint32_t c = threadIdx.x & 31, g = threadIdx.x >> 5;
    const uint64_t j = (uint64_t)blockIdx.x * 32 + c;
    double v[kReduceLoads];
#pragma unroll
    for (uint32_t k = 0; k < kReduceLoads; ++k) {
        const uint32_t r = g + 8u * k;
        v[k] = (j < n_out && r < n_ranges) ? partial[(uint64_t)r * n_out + j] : 0.0;
    }
    double s = 0.0;
#pragma unroll
    for (uint32_t k = 0; k < kReduceLoads; ++k)
        if (g + 8u * k < n_ranges) s += v[k];
    grp[g][c] = s;
    __syncthreads();
    if (g == 0 && j < n_out) {
        double t = grp[0][c];
#pragma unroll
        for (int k = 1; k < 8; ++k) t += grp[k][c];
        y[j] = t;
    }
}

}  // namespace

uint64_t gguf_values_read(int gguf_type, uint64_t data_len, uint64_t n_elems) {
    switch (gguf_type) {
        case kGgufF32: return data_len / 4;
        case kGgufF16: return data_len / 2;
        case kGgufQ4_0:
        case kGgufQ8_0: return n_elems;
        default: return 0;
    }
}

uint64_t gguf_blocks_ok(int gguf_type, uint64_t data_len, uint64_t n_elems) {
    const uint64_t bb = gguf_type == kGgufQ4_0 ? 18 : 34;
    const uint64_t whole = n_elems / 32;
    const uint64_t fit = data_len / bb;
    return whole < fit ? whole : fit;
}

cudaError_t read_tensor_f32(const void *data, uint64_t data_len, int gguf_type, uint64_t n_elems, float *out,
                            cudaStream_t st) {
    const uint64_t n = gguf_values_read(gguf_type, data_len, n_elems);
    if (n == 0) return cudaSuccess;
    switch (gguf_type) {
        case kGgufF32: return cudaMemcpyAsync(out, data, n * 4, cudaMemcpyDeviceToDevice, st);
        case kGgufF16: {
            const unsigned blocks = (unsigned)std::min<uint64_t>((n + 255) / 256, 148u * 16u);
            dequant_f16_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint16_t *>(data), n, out);
            return cudaGetLastError();
        }
        case kGgufQ4_0:
        case kGgufQ8_0: {
            const uint64_t ok = gguf_blocks_ok(gguf_type, data_len, n_elems);
            const uint64_t nb = (n_elems + 31) / 32;
            const unsigned blocks = (unsigned)((nb + 255) / 256);
            if (gguf_type == kGgufQ4_0)
                dequant_q_kernel<kGgufQ4_0><<<blocks, 256, 0, st>>>(static_cast<const uint8_t *>(data), ok, n_elems, out);
            else
                dequant_q_kernel<kGgufQ8_0><<<blocks, 256, 0, st>>>(static_cast<const uint8_t *>(data), ok, n_elems, out);
            return cudaGetLastError();
        }
        default: return cudaErrorInvalidValue;
    }
}

GemvPlan gemv_plan(uint64_t n_in, uint64_t n_out, uint64_t x_len, int num_sms, bool staged) {
    GemvPlan pl;
    pl.rows = x_len < n_in ? x_len : n_in;
    pl.staged = staged;
    const uint64_t cols = staged ? (uint64_t)kTileBlocks * 32 : (uint64_t)kCols;
    pl.col_tiles = (n_out + cols - 1) / cols;
    // at most one wave of CTAs at 4 per SM (the staged kernel's limit by
    // registers and by shared memory: a CTA more would run alone after the
    // wave), at least 64 rows a range, at most kMaxRanges ranges
    uint64_t ranges = (4ull * num_sms) / pl.col_tiles;
    const uint64_t by_rows = (pl.rows + 63) / 64;
    if (ranges > by_rows) ranges = by_rows;
    if (ranges > kMaxRanges) ranges = kMaxRanges;
    if (ranges < 1) ranges = 1;
    pl.rows_per_range = (pl.rows + ranges - 1) / ranges;
    pl.ranges = pl.rows_per_range ? (uint32_t)((pl.rows + pl.rows_per_range - 1) / pl.rows_per_range) : 1;
    return pl;
}

size_t gemv_workspace_bytes(uint64_t n_out) { return (size_t)kMaxRanges * n_out * sizeof(double); }

bool gemv_staged_ok(const void *w, uint64_t data_len, int gguf_type, uint64_t n_in, uint64_t n_out) {
    const bool quant = gguf_type == kGgufQ4_0 || gguf_type == kGgufQ8_0;
    const uint64_t n = n_in * n_out;
    const uint64_t have = quant ? gguf_blocks_ok(gguf_type, data_len, n) * 32 : gguf_values_read(gguf_type, data_len, n);
    return n_out % 256 == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 && have >= n;
}

namespace {

// Sets the dynamic shared-memory limit of `kernel` once per device.
template <typename K>
cudaError_t configure_once(K kernel, uint32_t smem, bool *configured) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && configured[dev]) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess && dev >= 0 && dev < 64) configured[dev] = true;
    return e;
}

// Launch with the programmatic-stream-serialisation attribute when
// `dependent`: the kernel may start before the previous kernel on the stream
// has ended, and waits for it at its griddepcontrol.wait.
template <typename... P, typename... A>
cudaError_t launch_ex(void (*kernel)(P...), dim3 grid, dim3 block, uint32_t smem, cudaStream_t st, bool dependent,
                      A... args) {
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = dependent ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int QT>
cudaError_t launch_staged(const uint8_t *w, uint64_t n_out, const GemvPlan &pl, const double *x, double *dst,
                          bool early, cudaStream_t st) {
    const dim3 grid((unsigned)pl.col_tiles, pl.ranges);
    if constexpr (QT == kGgufQ4_0) {
        static bool configured[64] = {false};
        const cudaError_t e = configure_once(gemv_q4_kernel, kQ4Smem, configured);
        if (e != cudaSuccess) return e;
        return launch_ex(gemv_q4_kernel, grid, dim3(kQ4Threads), kQ4Smem, st, early, w, n_out, pl.rows,
                         pl.rows_per_range, x, dst);
    } else {
        using Cf = StagedCfg<QT>;
        static bool configured[64] = {false};
        const cudaError_t e = configure_once(gemv_staged_kernel<QT>, Cf::SMEM, configured);
        if (e != cudaSuccess) return e;
        gemv_staged_kernel<QT><<<grid, kGemvThreads, Cf::SMEM, st>>>(w, n_out, pl.rows, pl.rows_per_range, x, dst);
        return cudaGetLastError();
    }
}

cudaError_t launch_reduce(const double *partial, uint32_t ranges, uint64_t n_out, double *y, cudaStream_t st) {
    return launch_ex(gemv_reduce_kernel, dim3((unsigned)((n_out + 31) / 32)), dim3(256), 0, st, true, partial, ranges,
                     n_out, y);
}

}  // namespace

cudaError_t gemv(const void *w, uint64_t data_len, int gguf_type, uint64_t n_in, uint64_t n_out, const double *x,
                 uint64_t x_len, double *y, double *partial, int num_sms, bool static_weights, cudaStream_t st) {
    const bool staged = gemv_staged_ok(w, data_len, gguf_type, n_in, n_out);
    const GemvPlan pl = gemv_plan(n_in, n_out, x_len, num_sms, staged);
    if (pl.rows == 0) return cudaMemsetAsync(y, 0, n_out * sizeof(double), st);
    uint64_t n_ok = 0;
    if (gguf_type == kGgufQ4_0 || gguf_type == kGgufQ8_0) {
        if (n_out % 32 != 0) return cudaErrorNotSupported;
        n_ok = gguf_blocks_ok(gguf_type, data_len, n_in * n_out);
    } else {
        n_ok = gguf_values_read(gguf_type, data_len, 0);
    }
    double *dst = pl.ranges == 1 ? y : partial;
    const dim3 grid((unsigned)pl.col_tiles, pl.ranges);
    const uint8_t *wb = static_cast<const uint8_t *>(w);
    if (staged) {
        cudaError_t se = cudaSuccess;
        switch (gguf_type) {
            case kGgufF32: se = launch_staged<kGgufF32>(wb, n_out, pl, x, dst, static_weights, st); break;
            case kGgufF16: se = launch_staged<kGgufF16>(wb, n_out, pl, x, dst, static_weights, st); break;
            case kGgufQ4_0: se = launch_staged<kGgufQ4_0>(wb, n_out, pl, x, dst, static_weights, st); break;
            case kGgufQ8_0: se = launch_staged<kGgufQ8_0>(wb, n_out, pl, x, dst, static_weights, st); break;
            default: return cudaErrorInvalidValue;
        }
        if (se != cudaSuccess || pl.ranges == 1) return se;
        return launch_reduce(partial, pl.ranges, n_out, y, st);
    }
    switch (gguf_type) {
        case kGgufF32: gemv_kernel<kGgufF32><<<grid, kGemvThreads, 0, st>>>(wb, n_ok, n_out, pl.rows, pl.rows_per_range, x, dst); break;
        case kGgufF16: gemv_kernel<kGgufF16><<<grid, kGemvThreads, 0, st>>>(wb, n_ok, n_out, pl.rows, pl.rows_per_range, x, dst); break;
        case kGgufQ4_0: gemv_kernel<kGgufQ4_0><<<grid, kGemvThreads, 0, st>>>(wb, n_ok, n_out, pl.rows, pl.rows_per_range, x, dst); break;
        case kGgufQ8_0: gemv_kernel<kGgufQ8_0><<<grid, kGemvThreads, 0, st>>>(wb, n_ok, n_out, pl.rows, pl.rows_per_range, x, dst); break;
        default: return cudaErrorInvalidValue;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || pl.ranges == 1) return e;
    return launch_reduce(partial, pl.ranges, n_out, y, st);
}

}  // namespace bml
