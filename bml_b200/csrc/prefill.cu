// prefill.cu -- causal GQA prefill attention on tcgen05 tensor cores (sm_100a).
//
// Computes, for every token t of every prompt, the attention block of
// forward_layer_cached (crates/compiler/src/gguf_compiler.rs:1008-1050 in
// SugarFreeDoNoSo/bml) over positions [0, t] -- which is what the reference's
// forward_cached token loop (gguf_compiler.rs:946-958) does one token at a
// time.  Here the whole prompt runs at once as a flash-attention kernel:
// bf16/f16 operands, f32 accumulation, online softmax.
//
// One CTA handles two consecutive 128-row query tiles, A and B, of one
// (sequence, q head).  Both read the same K/V tiles, so every K/V tile in
// shared memory feeds twice the tensor-core work, and while the softmax of
// one tile runs the tensor core works on the other.  Tensor memory (512
// columns) holds S_A, S_B (128 columns each) and the accumulators O_A, O_B.
// Warp roles:
//   warp 0      TMA producer: Q_A and Q_B once, then K and V tiles of 128
//               positions into a stage ring (cp.async.bulk.tensor, 128B
//               swizzle, no multicast), completing on mbarriers.
//   warp 1      allocates tensor memory; lane 0 issues every tcgen05.mma.
//   warps 2-5   softmax of tile A, warps 6-9 softmax of tile B: thread r
//               owns query row r (TMEM lane r).  It loads its 128 scores
//               from tensor memory at once, writes P back over S as packed
//               16-bit pairs with tcgen05.st in two halves (P.V starts on the
//               first half while the second is computed),
//               and rescales O in TMEM only when its running max grew by
//               more than 2^8 (the final O / l is exact for any fixed
//               reference max).
// P.V takes P straight from tensor memory (tcgen05.mma with the A operand in
// TMEM) and V from shared memory.  The MMA issue order per K/V tile j is
// PV_A(j), S_A(j+1), PV_B(j), S_B(j+1).  Tensor-core operations of one
// thread run in issue order, so S_X(j+1) overwrites P_X(j) only after PV_X(j)
// has read it, and the commit that announces S_X(j+1) also tells the softmax
// that PV_X(j) has finished: O_X may be rescaled and P_X rewritten.
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>

#include "prefill.cuh"

namespace bml {

namespace {

constexpr int BM = 128;  // query rows per tile (TMEM lanes)
constexpr int BN = 128;  // kv positions per tile
constexpr int kThreads = 320;  // producer, MMA issuer, 4 + 4 softmax warps
constexpr int kMaxStages = 4;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// The MMA warp tests the barriers of its next block of MMAs this many MMAs
// before the end of the current block.
constexpr int kGateLookahead = 1;

template <int D>
struct PCfg {
    static constexpr int KB = D / 64;                // 128-byte column blocks of a row
    static constexpr int Q_BYTES = BM * D * 2;       // one Q tile
    static constexpr int TILE_BYTES = BN * D * 2;    // one K or V tile
    static constexpr int STAGES = D == 128 ? 2 : 4;
    static constexpr int OFF_Q = 0;                  // Q_A, Q_B
    static constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
    static constexpr int OFF_V = OFF_K + STAGES * TILE_BYTES;
    static constexpr int OFF_BAR = OFF_V + STAGES * TILE_BYTES;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;  // + alignment slack
    // tensor memory: S_x at x*128 (P_x aliases its first 64 columns),
    // O_x at 256 + x*D
    static constexpr uint32_t O_COL0 = 256;
    static constexpr uint32_t TMEM_COLS = 512;
};
static_assert(PCfg<128>::SMEM <= 227 * 1024, "shared memory");
static_assert(PCfg<64>::SMEM <= 227 * 1024, "shared memory");
static_assert(PCfg<64>::STAGES <= kMaxStages && PCfg<128>::STAGES <= kMaxStages, "stages");

struct PrefillParams {
    CUtensorMap tq, tk, tv;  // 3-D maps (d, heads, n_seqs*seq_len), box (64, 1, 128)
    void *out;
    uint32_t *err;
    uint32_t S, H, Hkv, n_seqs, n_mtiles, n_pairs;
    float scale_log2;  // scale * log2(e)
    int causal;
    int out_f32;
};

// ----------------------------------------------------------------- PTX
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// true in exactly one lane of a converged warp
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, e;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]; A is M x 16 with two 16-bit
// elements per 32-bit column (8 columns per instruction).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
        "%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *w) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16};" ::"r"(taddr),
        "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]), "r"(w[8]),
        "r"(w[9]), "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]), "r"(w[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, 128B swizzle, sm_100 version bits.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor for kind::f16: f32 accumulate, A K-major.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t in_fmt, uint32_t m, uint32_t n, uint32_t b_mn_major) {
    return (1u << 4) | (in_fmt << 7) | (in_fmt << 10) | (b_mn_major << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// (2^e.x, 2^e.y) on the FMA pipe, for a share of the softmax's
// exponentials (the SFU's exp2 runs at 16 a clock an SM, which is as long
// per 128 x 128 tile as the tile's two MMAs).  Range reduction e = n + f,
// n = round(e) by the 1.5 * 2^23 add, f in [-1/2, 1/2]; 2^f by a cubic
// fitted here by reweighted least squares on Chebyshev nodes (maximum
// relative error 7.7e-5 on [-1/2, 1/2], below bf16's 2^-8 rounding of p);
// 2^n added to the exponent field as an integer.  Arguments below -120
// (masked keys are -inf) give 2^-120 instead of 0: ~1e-36 of a row sum of
// at least 1.
__device__ __forceinline__ float2 exp2_poly_pair(float2 e) {
    e.x = fmaxf(e.x, -120.f);
    e.y = fmaxf(e.y, -120.f);
    const float2 t = __fadd2_rn(e, make_float2(12582912.f, 12582912.f));  // low mantissa bits: round(e)
    const float2 r = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
    const float2 f = __ffma2_rn(r, make_float2(-1.f, -1.f), e);            // e - round(e), exact
    float2 q = __ffma2_rn(f, make_float2(0.055088736f, 0.055088736f), make_float2(0.24260406f, 0.24260406f));
    q = __ffma2_rn(f, q, make_float2(0.69327623f, 0.69327623f));
    q = __ffma2_rn(f, q, make_float2(0.99992895f, 0.99992895f));
    q.x = __int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23));
    q.y = __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23));
    return q;
}

// two f32 -> one 32-bit word of 16-bit values, lo in the low half
template <bool kF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if (kF16) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&h);
    }
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// ----------------------------------------------------------------- kernel
template <int D, bool kF16>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
    using C = PCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128B-swizzle atoms
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t *sQ = smem + C::OFF_Q;
    uint8_t *sK = smem + C::OFF_K;
    uint8_t *sV = smem + C::OFF_V;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *q_full = bars;                    // Q_A and Q_B landed
    uint64_t *k_full = bars + 1;                // [stage]
    uint64_t *k_empty = k_full + kMaxStages;    // [stage]
    uint64_t *v_full = k_empty + kMaxStages;    // [stage]
    uint64_t *v_empty = v_full + kMaxStages;    // [stage]
    uint64_t *s_full = v_empty + kMaxStages;    // [chain]: S of the chain's current tile in TMEM
    uint64_t *p_full = s_full + 2;              // [chain][half]: P columns 32*half.. of the chain's tile in TMEM
    uint64_t *o_final = p_full + 4;             // [chain]: last P.V of the chain done
    volatile uint32_t *misc = reinterpret_cast<volatile uint32_t *>(o_final + 2);  // [0] tmem base, [1] abort

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // work unit: heaviest (last) tile pairs first
    const uint32_t per = p.n_seqs * p.H;
    const uint32_t pair = p.n_pairs - 1 - blockIdx.x / per;
    const uint32_t bh = blockIdx.x % per;
    const uint32_t b = bh / p.H, h = bh % p.H;
    const uint32_t hk = h / (p.H / p.Hkv);
    const uint32_t kv_tiles_all = (p.S + BN - 1) / BN;
    // Query tile of each chain and its number of K/V tiles.  BM == BN, so
    // causally tile m sees K/V tiles 0..m.  nt1 >= nt0: chain B is always
    // the last user of a K/V stage.  (With an odd tile count the last pair's
    // tile B lies past the prompt; it runs on whatever rows the map returns
    // and writes nothing.)
    const uint32_t mt0 = 2 * pair, mt1 = 2 * pair + 1;
    const uint32_t nt0 = p.causal ? min(kv_tiles_all, mt0 + 1) : kv_tiles_all;
    const uint32_t nt1 = p.causal ? min(kv_tiles_all, mt1 + 1) : kv_tiles_all;
    const int row_base = (int)(b * p.S);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < C::STAGES; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int x = 0; x < 2; ++x) {
            mbar_init(&s_full[x], 1);
            mbar_init(&p_full[2 * x], 4);
            mbar_init(&p_full[2 * x + 1], 4);
            mbar_init(&o_final[x], 1);
        }
        misc[1] = 0u;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.tq);
        prefetch_tmap(&p.tk);
        prefetch_tmap(&p.tv);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32((const void *)&misc[0])),
                     "r"(C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];
    volatile uint32_t *abort_flag = misc + 1;

    if (warp == 0) {
        // ------------------------------------------------------------- TMA producer
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
#pragma unroll
            for (int x = 0; x < 2; ++x)
#pragma unroll
                for (int kb = 0; kb < C::KB; ++kb)
                    tma_load_3d(sQ + x * C::Q_BYTES + kb * BM * 128, &p.tq, kb * 64, (int)h,
                                row_base + (int)((x ? mt1 : mt0) * BM), q_full);
            for (uint32_t j = 0; j < nt1; ++j) {
                const uint32_t st = j % C::STAGES, u = j / C::STAGES;
                const int row = row_base + (int)(j * BN);
                if (j >= (uint32_t)C::STAGES) mbar_wait(&k_empty[st], (u & 1u) ^ 1u, abort_flag, p.err);
                mbar_arrive_expect_tx(&k_full[st], C::TILE_BYTES);
#pragma unroll
                for (int kb = 0; kb < C::KB; ++kb)
                    tma_load_3d(sK + st * C::TILE_BYTES + kb * BN * 128, &p.tk, kb * 64, (int)hk, row, &k_full[st]);
                if (j >= (uint32_t)C::STAGES) mbar_wait(&v_empty[st], (u & 1u) ^ 1u, abort_flag, p.err);
                mbar_arrive_expect_tx(&v_full[st], C::TILE_BYTES);
#pragma unroll
                for (int kb = 0; kb < C::KB; ++kb)
                    tma_load_3d(sV + st * C::TILE_BYTES + kb * BN * 128, &p.tv, kb * 64, (int)hk, row, &v_full[st]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        // The whole warp runs this loop converged and one elected lane issues
        // each tcgen05 instruction.  The tensor core queues only about one MMA
        // ahead, so every cycle spent between two MMAs beyond that is lost;
        // measured on B200, barrier tests cost a single issuing thread (in a
        // divergent branch) up to ~35 cycles per MMA while the softmax warps
        // run beside it, and next to nothing for a converged warp.  Each block
        // of MMAs also tests the barriers of the next block before its own last
        // MMA and blocks on them only if they were not complete yet.
        constexpr uint32_t fmt = kF16 ? 0u : 1u;
        constexpr uint32_t idesc_qk = make_idesc(fmt, BM, BN, 0);
        constexpr uint32_t idesc_pv = make_idesc(fmt, BM, D, 1);
        // Base descriptors; an operand `bytes` further on is the base plus
        // bytes >> 4 (the 14-bit start field never carries: shared memory
        // addresses stay below 256 KB).
        const uint64_t dq = smem_desc(smem_u32(sQ), 16, 1024);
        const uint64_t dk = smem_desc(smem_u32(sK), 16, 1024);
        const uint64_t dv = smem_desc(smem_u32(sV), BN * 128, 1024);
        struct Gate {  // one or two barrier phases; b1 may be null
            uint64_t *b0;
            uint32_t p0;
            uint64_t *b1;
            uint32_t p1;
        };
        auto gate_test = [&](const Gate &g) {
            bool ok = g.b0 == nullptr || mbar_test_wait(g.b0, g.p0);
            if (g.b1) ok = ok & mbar_test_wait(g.b1, g.p1);
            return ok;
        };
        auto gate_wait = [&](const Gate &g, bool ready) {
            if (!ready) {
                if (g.b0) mbar_wait(g.b0, g.p0, abort_flag, p.err);
                if (g.b1) mbar_wait(g.b1, g.p1, abort_flag, p.err);
            }
            __syncwarp();
            tc_fence_after();
        };
        // S_x = Q_x K(j)^T.  Chain B, the last user of K(j), releases the stage.
        auto qk = [&](uint32_t x, uint32_t j, const Gate &next) {
            const uint32_t st = j % C::STAGES;
            const uint64_t a0 = dq + ((x * C::Q_BYTES) >> 4);
            const uint64_t b0 = dk + ((st * C::TILE_BYTES) >> 4);
            const uint32_t d = tmem + x * 128;
            bool ready = true;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                if (kk == D / 16 - kGateLookahead) ready = gate_test(next);
                // k-step kk: 128B column block kk/4, 32 bytes per step inside it (BM == BN)
                const uint32_t off = ((kk >> 2) * (BM * 128) + (kk & 3) * 32) >> 4;
                if (elect_one()) tc_mma_ss(d, a0 + off, b0 + off, idesc_qk, kk > 0);
                __syncwarp();
            }
            if (elect_one()) {
                tc_commit(&s_full[x]);
                if (x == 1) tc_commit(&k_empty[st]);
            }
            __syncwarp();
            return ready;
        };
        // O_x += P_x V(j) over kv rows 64h..64h+63, P_x read from tensor
        // memory (over S_x).  The softmax releases P in these two halves,
        // so the first half of P.V overlaps the second half of its work.
        auto pv = [&](uint32_t x, uint32_t j, int h, const Gate &next) {
            const uint32_t st = j % C::STAGES;
            const uint64_t b0 = dv + ((st * C::TILE_BYTES) >> 4);
            const uint32_t d = tmem + C::O_COL0 + x * D, a = tmem + x * 128;
            bool ready = true;
#pragma unroll
            for (int k4 = 0; k4 < BN / 32; ++k4) {
                const int kk = h * (BN / 32) + k4;  // 16 kv rows of 128 B per step
                if (k4 == BN / 32 - kGateLookahead) ready = gate_test(next);
                if (elect_one())
                    tc_mma_ts(d, a + kk * 8, b0 + ((kk * 16 * 128) >> 4), idesc_pv, (kk > 0 || j > 0) ? 1u : 0u);
                __syncwarp();
            }
            if (h == 1 && elect_one()) {
                if (x == 1) tc_commit(&v_empty[st]);
                if (j + 1 == (x ? nt1 : nt0)) tc_commit(&o_final[x]);
            }
            __syncwarp();
            return ready;
        };
        // gate of the first P.V block of iteration j: chain A's while it runs
        // (chain A is then the first user of V(j)), else chain B's
        auto gate_pv0 = [&](uint32_t j) {
            const uint32_t st = j % C::STAGES, ph = (j / C::STAGES) & 1u;
            return Gate{&p_full[j < nt0 ? 0 : 2], j & 1u, &v_full[st], ph};
        };
        const Gate none = {nullptr, 0u, nullptr, 0u};

        gate_wait(Gate{q_full, 0u, &k_full[0], 0u}, false);
        qk(0, 0, none);
        gate_wait(gate_pv0(0), qk(1, 0, gate_pv0(0)));
        for (uint32_t j = 0; j < nt1; ++j) {
            const uint32_t jp = j & 1u;
            const uint32_t st1 = (j + 1) % C::STAGES, ph1 = ((j + 1) / C::STAGES) & 1u;
            if (j < nt0) {
                {
                    const Gate g = {&p_full[1], jp, nullptr, 0u};
                    gate_wait(g, pv(0, j, 0, g));
                }
                if (j + 1 < nt0) {
                    const Gate g2 = {&k_full[st1], ph1, nullptr, 0u};
                    gate_wait(g2, pv(0, j, 1, g2));
                    const Gate g3 = {&p_full[2], jp, nullptr, 0u};
                    gate_wait(g3, qk(0, j + 1, g3));
                } else {
                    const Gate g2 = {&p_full[2], jp, nullptr, 0u};
                    gate_wait(g2, pv(0, j, 1, g2));
                }
            }
            {
                const Gate g = {&p_full[3], jp, nullptr, 0u};
                gate_wait(g, pv(1, j, 0, g));
            }
            if (j + 1 < nt1) {
                const Gate g5 = (j + 1 >= nt0) ? Gate{&k_full[st1], ph1, nullptr, 0u} : none;
                gate_wait(g5, pv(1, j, 1, g5));
                const Gate g6 = gate_pv0(j + 1);
                gate_wait(g6, qk(1, j + 1, g6));
            } else {
                pv(1, j, 1, none);
            }
        }
    } else {
        // ------------------------------------------------------------- softmax
        const uint32_t x = (uint32_t)(warp - 2) >> 2;  // chain: 0 = tile A (warps 2-5), 1 = tile B (6-9)
        const uint32_t q4 = warp & 3;                   // TMEM lane quarter of this warp
        const uint32_t r = q4 * 32 + lane;              // query row within the tile
        const uint32_t t = (x ? mt1 : mt0) * BM + r;    // query position
        const uint32_t nt = x ? nt1 : nt0;
        const uint32_t lane_addr = (q4 * 32) << 16;
        const uint32_t s_col = tmem + lane_addr + x * 128;
        const uint32_t o_col = tmem + lane_addr + C::O_COL0 + x * D;
        const float c = p.scale_log2;
        const uint32_t lim = p.causal ? t : p.S - 1;  // last key this row sees
        float m_run = -INFINITY, l_run = 0.f;

        for (uint32_t j = 0; j < nt; ++j) {
            mbar_wait(&s_full[x], j & 1u, abort_flag, p.err);
            __syncwarp();  // lanes leave the spin separately; tcgen05.ld needs the whole warp
            tc_fence_after();
            const uint32_t kv0 = j * BN;
            const bool mask_tile = kv0 + BN - 1 > lim;

            // all 128 scores of the row in one round trip
            float sv[BN];
#pragma unroll
            for (int cc = 0; cc < BN / 32; ++cc) tmem_ld32(s_col + cc * 32, sv + cc * 32);
            tmem_wait_ld();
            if (mask_tile) {
#pragma unroll
                for (int i = 0; i < BN; ++i)
                    if (kv0 + i > lim) sv[i] = -INFINITY;
            }
            // row max: 8 independent chains of three-input max
            float mx8[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                float a = fmax3(sv[k], sv[k + 8], sv[k + 16]);
#pragma unroll
                for (int i = 24; i < BN - 8; i += 16) a = fmax3(a, sv[k + i], sv[k + i + 8]);  // up to k+112
                mx8[k] = fmaxf(a, sv[k + BN - 8]);                                              // k+120
            }
            const float mh = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
            const float m_tile = mh * c;
            float m_new = m_run;
            if (m_run == -INFINITY || m_tile > m_run + kRescaleThreshold) m_new = fmaxf(m_run, m_tile);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            const float alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_use);
            const bool rescale = (j > 0) && (m_new != m_run);
            m_run = m_new;

            // p = 2^(s*c - m), written as packed 16-bit pairs into columns
            // 0..63 of S_x (kv 2i, 2i+1 -> column i) and released to the MMA
            // warp in two halves.  An eighth of the exponentials run on the FMA
            // pipe (exp2_poly_pair), the rest on the SFU: measured on B200
            // (4 x 8192 tokens, kernel alone), 2.002 ms with none, 1.910 with
            // an eighth, 1.910-1.922 with 3/16, 1.926-1.957 with a quarter,
            // 2.14 with 3/8 and 2.21 with half (issue slots run out).
            const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_use, -m_use);
            float2 sum4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};
#pragma unroll
            for (int hv = 0; hv < 2; ++hv) {
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                    const int qc = hv * 2 + q2;
                    uint32_t w[16];
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        float2 e = __ffma2_rn(make_float2(sv[qc * 32 + i], sv[qc * 32 + i + 1]), c2, nm2);
                        if (((i >> 1) & 7) == 7) {  // an eighth of the pairs on the FMA pipe
                            e = exp2_poly_pair(e);
                        } else {
                            e.x = fast_exp2(e.x);
                            e.y = fast_exp2(e.y);
                        }
                        sum4[(i >> 1) & 3] = __fadd2_rn(sum4[(i >> 1) & 3], e);
                        w[i >> 1] = pack2<kF16>(e.x, e.y);
                    }
                    tmem_st16(s_col + qc * 16, w);
                }
                if (hv == 0 && __any_sync(0xffffffffu, rescale)) {
                    // O rescale (rare), before P.V(j) accumulates into O_x and
                    // after half of the scores are dead.  PV_x(j-1) has
                    // finished: S_x(j) was issued after it and its commit covers
                    // every earlier MMA.
                    const float a = rescale ? alpha : 1.f;
#pragma unroll
                    for (int cc = 0; cc < D / 32; ++cc) {
                        float o[32];
                        tmem_ld32(o_col + cc * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= a;
                        tmem_st32(o_col + cc * 32, o);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[2 * x + hv]);
            }
            const float2 sum2 = __fadd2_rn(__fadd2_rn(sum4[0], sum4[1]), __fadd2_rn(sum4[2], sum4[3]));
            l_run = l_run * alpha + (sum2.x + sum2.y);
        }

        // epilogue: O / l -> global
        mbar_wait(&o_final[x], 0, abort_flag, p.err);
        __syncwarp();
        tc_fence_after();
        const float inv_l = 1.f / l_run;
        const bool valid = t < p.S;
        const size_t orow = ((size_t)(row_base + t) * p.H + h) * D;
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
            float o[32];
            tmem_ld32(o_col + cc * 32, o);
            tmem_wait_ld();
            if (valid) {
                if (p.out_f32) {
                    float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + orow + cc * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        dst[i] = make_float4(o[4 * i] * inv_l, o[4 * i + 1] * inv_l, o[4 * i + 2] * inv_l,
                                             o[4 * i + 3] * inv_l);
                } else {
                    uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.out) + orow + cc * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[i] = make_uint4(pack2<kF16>(o[8 * i] * inv_l, o[8 * i + 1] * inv_l),
                                            pack2<kF16>(o[8 * i + 2] * inv_l, o[8 * i + 3] * inv_l),
                                            pack2<kF16>(o[8 * i + 4] * inv_l, o[8 * i + 5] * inv_l),
                                            pack2<kF16>(o[8 * i + 6] * inv_l, o[8 * i + 7] * inv_l));
                }
            }
        }
        tc_fence_before();
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS)
                     : "memory");
    }
}

// ----------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 3-D view (d, heads, rows) of a [rows][heads][d] 16-bit tensor; box (64, 1, 128).
bool make_map(CUtensorMap *map, const void *base, bool f16, uint32_t d, uint32_t heads, uint64_t rows) {
    auto enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[3] = {d, heads, rows};
    cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)d * heads * 2};
    cuuint32_t box[3] = {64, 1, 128};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                     const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int D, bool kF16>
cudaError_t launch_t(const PrefillParams &p, unsigned grid, cudaStream_t stream) {
    using C = PCfg<D>;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(prefill_kernel<D, kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::SMEM);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    prefill_kernel<D, kF16><<<grid, kThreads, C::SMEM, stream>>>(p);
    return cudaGetLastError();
}

__device__ uint32_t g_prefill_err;

// Device address of the prefill error word on the current device.
uint32_t *prefill_err_word() {
    static std::mutex mu;
    static uint32_t *addr[64] = {nullptr};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_prefill_err) == cudaSuccess) addr[dev] = static_cast<uint32_t *>(ptr);
    }
    return addr[dev];
}

}  // namespace

cudaError_t launch_prefill(const PrefillArgs &a, cudaStream_t stream) {
    const bool f16 = a.in_dtype == BML_F16;
    const uint64_t rows = (uint64_t)a.n_seqs * a.seq_len;
    if (rows > 0x7fffffffull) return cudaErrorInvalidValue;
    static thread_local PrefillParams p;
    if (!make_map(&p.tq, a.q, f16, a.head_dim, a.n_heads, rows) ||
        !make_map(&p.tk, a.k, f16, a.head_dim, a.n_kv, rows) ||
        !make_map(&p.tv, a.v, f16, a.head_dim, a.n_kv, rows))
        return cudaErrorInvalidValue;
    p.out = a.out;
    p.err = prefill_err_word();
    p.S = a.seq_len;
    p.H = a.n_heads;
    p.Hkv = a.n_kv;
    p.n_seqs = a.n_seqs;
    p.n_mtiles = (a.seq_len + BM - 1) / BM;
    p.n_pairs = (p.n_mtiles + 1) / 2;
    p.scale_log2 = (float)((double)a.scale * 1.4426950408889634);
    p.causal = a.causal ? 1 : 0;
    p.out_f32 = a.out_dtype == BML_F32 ? 1 : 0;
    const uint64_t grid = (uint64_t)p.n_pairs * a.n_seqs * a.n_heads;
    if (grid == 0 || grid > 0x7fffffffull) return cudaErrorInvalidValue;
    switch (a.head_dim) {
        case 64: return f16 ? launch_t<64, true>(p, (unsigned)grid, stream) : launch_t<64, false>(p, (unsigned)grid, stream);
        case 128:
            return f16 ? launch_t<128, true>(p, (unsigned)grid, stream) : launch_t<128, false>(p, (unsigned)grid, stream);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace bml
