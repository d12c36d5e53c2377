// prefill.cu -- causal GQA prefill attention on tcgen05 tensor cores (sm_100a).
//
// Computes, for every token t of every prompt, the attention block of
// forward_layer_cached (crates/compiler/src/gguf_compiler.rs:1008-1050 in
// SugarFreeDoNoSo/bml) over positions [0, t] -- which is what the reference's
// forward_cached token loop (gguf_compiler.rs:946-958) does one token at a
// time.  Here the whole prompt runs at once as a flash-attention kernel:
// bf16/f16 operands, f32 accumulation, online softmax.
//
// One CTA handles 128 query rows of one (sequence, q head).  Warp roles:
//   warp 0      TMA producer: Q once, then K and V tiles of 128 positions
//               into a multi-stage ring (cp.async.bulk.tensor, 128B swizzle,
//               no multicast), completing on mbarriers.
//   warp 1      allocates tensor memory; lane 0 issues every tcgen05.mma:
//               S = Q K^T into one of two TMEM S buffers, and O += P V into
//               the TMEM O accumulator; tcgen05.commit signals completion.
//   warps 2-5   softmax: thread r owns query row r (TMEM lane r).  It reads
//               its S row with tcgen05.ld, applies the causal mask, keeps the
//               running max / sum, writes P (bf16) into 128B-swizzled shared
//               memory for the next MMA, and rescales O in TMEM only when its
//               running max grew by more than 2^8 (the final O / l is exact
//               for any fixed reference max).  At the end it divides O by l.
// The MMA warp issues S(j+1) = Q K(j+1)^T before waiting for P(j), so the
// tensor core computes the next scores while the softmax warps work.
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>

#include "prefill.cuh"

namespace bml {

namespace {

constexpr int BM = 128;  // query rows per CTA (TMEM lanes)
constexpr int BN = 128;  // kv positions per tile
constexpr int kThreads = 320;  // producer, MMA issuer, 8 softmax warps
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct PCfg {
    static constexpr int KB = D / 64;                // 128-byte column blocks of a row
    static constexpr int Q_BYTES = BM * D * 2;
    static constexpr int TILE_BYTES = BN * D * 2;
    static constexpr int P_BYTES = BM * BN * 2;
    static constexpr int STAGES = D == 128 ? 2 : 3;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + Q_BYTES;
    static constexpr int OFF_V = OFF_K + STAGES * TILE_BYTES;
    static constexpr int OFF_P = OFF_V + STAGES * TILE_BYTES;
    static constexpr int OFF_BAR = OFF_P + P_BYTES;
    // row-max exchange [2 buffers][2 halves][BM] + row-sum exchange [2 halves][BM]
    static constexpr int OFF_X = OFF_BAR + 256;
    static constexpr int SMEM = OFF_X + 3 * 2 * BM * 4 + 1024;  // + alignment slack
    static constexpr uint32_t S_COL = 0;    // two S buffers: columns [0,128), [128,256)
    static constexpr uint32_t O_COL = 256;  // O: columns [256, 256+D)
    static constexpr uint32_t TMEM_COLS = 512;
};

struct PrefillParams {
    CUtensorMap tq, tk, tv;  // 3-D maps (d, heads, n_seqs*seq_len), box (64, 1, 128)
    void *out;
    uint32_t *err;
    uint32_t S, H, Hkv, n_seqs, n_mtiles;
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

// 32 consecutive f32 columns of this thread's TMEM lane.
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

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor, 128B swizzle, sm_100 version bits.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor for kind::f16: f32 accumulate, A K-major.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t in_fmt, uint32_t m, uint32_t n, uint32_t b_mn_major) {
    return (1u << 4) | (in_fmt << 7) | (in_fmt << 10) | (b_mn_major << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
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
    uint8_t *sP = smem + C::OFF_P;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *q_full = bars;
    uint64_t *k_full = bars + 1;
    uint64_t *k_empty = k_full + C::STAGES;
    uint64_t *v_full = k_empty + C::STAGES;
    uint64_t *v_empty = v_full + C::STAGES;
    uint64_t *s_full = v_empty + C::STAGES;  // [2]
    uint64_t *s_empty = s_full + 2;          // [2]
    uint64_t *p_full = s_empty + 2;
    uint64_t *o_done = p_full + 1;
    volatile uint32_t *misc = reinterpret_cast<volatile uint32_t *>(o_done + 1);  // [0] tmem base, [1] abort

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // work unit: heaviest (last) query tiles first
    const uint32_t per = p.n_seqs * p.H;
    const uint32_t mt = p.n_mtiles - 1 - blockIdx.x / per;
    const uint32_t bh = blockIdx.x % per;
    const uint32_t b = bh / p.H, h = bh % p.H;
    const uint32_t hk = h / (p.H / p.Hkv);
    const uint32_t q0 = mt * BM;
    const uint32_t kv_tiles_all = (p.S + BN - 1) / BN;
    const uint32_t n_tiles = p.causal ? min(kv_tiles_all, (q0 + BM - 1) / BN + 1) : kv_tiles_all;
    const int row_base = (int)(b * p.S);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < C::STAGES; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_empty[i], 8);
        }
        mbar_init(p_full, 8);
        mbar_init(o_done, 1);
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
            mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
            for (int kb = 0; kb < C::KB; ++kb)
                tma_load_3d(sQ + kb * BM * 128, &p.tq, kb * 64, (int)h, row_base + (int)q0, q_full);
            for (uint32_t j = 0; j < n_tiles; ++j) {
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
        if (lane == 0) {
            constexpr uint32_t fmt = kF16 ? 0u : 1u;
            constexpr uint32_t idesc_qk = make_idesc(fmt, BM, BN, 0);
            constexpr uint32_t idesc_pv = make_idesc(fmt, BM, D, 1);
            const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV),
                           p_base = smem_u32(sP);
            mbar_wait(q_full, 0, abort_flag, p.err);
            auto issue_qk = [&](uint32_t j) {
                const uint32_t st = j % C::STAGES, sb = j & 1u;
                mbar_wait(&k_full[st], (j / C::STAGES) & 1u, abort_flag, p.err);
                if (j >= 2) mbar_wait(&s_empty[sb], ((j >> 1) & 1u) ^ 1u, abort_flag, p.err);
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
                    const uint32_t koff = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
                    tc_mma_ss(tmem + C::S_COL + sb * BN, smem_desc(q_base + off, 16, 1024),
                              smem_desc(k_base + st * C::TILE_BYTES + koff, 16, 1024), idesc_qk, kk > 0);
                }
                tc_commit(&s_full[sb]);
                tc_commit(&k_empty[st]);
            };
            issue_qk(0);
            for (uint32_t j = 0; j < n_tiles; ++j) {
                if (j + 1 < n_tiles) issue_qk(j + 1);
                const uint32_t st = j % C::STAGES;
                mbar_wait(p_full, j & 1u, abort_flag, p.err);
                mbar_wait(&v_full[st], (j / C::STAGES) & 1u, abort_flag, p.err);
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    const uint32_t poff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
                    const uint32_t voff = kk * 16 * 128;  // 16 kv rows of 128 B
                    tc_mma_ss(tmem + C::O_COL, smem_desc(p_base + poff, 16, 1024),
                              smem_desc(v_base + st * C::TILE_BYTES + voff, BN * 128, 1024), idesc_pv,
                              (j > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(o_done);
                tc_commit(&v_empty[st]);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------- softmax
        // Two warps share each TMEM lane quarter: warp w owns rows
        // 32*(w%4) .. +31 and the column half hf of every S row (and of O);
        // the pair exchanges its half-row maxima once per tile.
        const uint32_t q4 = warp & 3;            // TMEM lane quarter of this warp
        const uint32_t hf = (warp - 2) >> 2;     // column half: 0 for warps 2-5, 1 for 6-9
        const uint32_t r = q4 * 32 + lane;       // query row within the tile
        const uint32_t t = q0 + r;               // query position
        const uint32_t lane_addr = (q4 * 32) << 16;
        constexpr int HC = BN / 2;               // score columns per thread
        constexpr int HD = D / 2;                // output columns per thread
        float *xch = reinterpret_cast<float *>(smem + C::OFF_X);  // [buf][half][row]
        const float c = p.scale_log2;
        float m_run = -INFINITY, l_part = 0.f;
        uint8_t *prow = sP + (r >> 3) * 1024 + (r & 7) * 128 + hf * (BM * 128);

        for (uint32_t j = 0; j < n_tiles; ++j) {
            const uint32_t sb = j & 1u;
            mbar_wait(&s_full[sb], (j >> 1) & 1u, abort_flag, p.err);
            __syncwarp();  // lanes leave the spin separately; tcgen05.ld needs the whole warp
            tc_fence_after();
            float s[HC];
#pragma unroll
            for (int cc = 0; cc < HC / 32; ++cc)
                tmem_ld32(tmem + lane_addr + C::S_COL + sb * BN + hf * HC + cc * 32, s + cc * 32);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[sb]);

            const uint32_t kv0 = j * BN + hf * HC;   // key position of s[0]
            if (p.causal) {
                if (kv0 + HC - 1 > t) {
#pragma unroll
                    for (int i = 0; i < HC; ++i)
                        if (kv0 + i > t) s[i] = -INFINITY;
                }
            } else if (kv0 + HC > p.S) {
#pragma unroll
                for (int i = 0; i < HC; ++i)
                    if (kv0 + i >= p.S) s[i] = -INFINITY;
            }
            // half-row max: 8 chains of three-input max over 64 columns
            float mx8[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                float a = fmax3(s[k], s[k + 8], s[k + 16]);
#pragma unroll
                for (int i = 24; i + 8 < HC; i += 16) a = fmax3(a, s[k + i], s[k + i + 8]);  // up to k+48
                mx8[k] = fmaxf(a, s[k + HC - 8]);                                           // k+56
            }
            float mh = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
            // exchange with the partner warp (double-buffered by tile parity)
            xch[(sb * 2 + hf) * BM + r] = mh;
            __syncwarp();
            named_bar_sync(2 + q4, 64);
            mh = fmaxf(mh, xch[(sb * 2 + (hf ^ 1u)) * BM + r]);
            const float m_tile = mh * c;
            float m_new = m_run;
            if (m_run == -INFINITY || m_tile > m_run + kRescaleThreshold) m_new = fmaxf(m_run, m_tile);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            const float alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_use);
            // p = 2^(s*c - m): one pair in four on the FMA/ALU pipes, the rest
            // on the SFU; summed in 4 independent packed chains
            const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_use, -m_use);
            float2 sum4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};
#pragma unroll
            for (int i = 0; i < HC; i += 2) {
                float2 x = __ffma2_rn(make_float2(s[i], s[i + 1]), c2, nm2);
                if (((i >> 1) & 3) == 3) {
                    x = exp2_poly2(x);
                } else {
                    x.x = fast_exp2(x.x);
                    x.y = fast_exp2(x.y);
                }
                s[i] = x.x;
                s[i + 1] = x.y;
                sum4[(i >> 1) & 3] = __fadd2_rn(sum4[(i >> 1) & 3], x);
            }
            const float2 sum2 = __fadd2_rn(__fadd2_rn(sum4[0], sum4[1]), __fadd2_rn(sum4[2], sum4[3]));
            l_part = l_part * alpha + (sum2.x + sum2.y);
            const bool rescale = (j > 0) && (m_new != m_run);
            m_run = m_new;

            if (j > 0) {
                // PV(j-1) must be done: it reads P, and O gets rescaled here
                mbar_wait(o_done, (j - 1) & 1u, abort_flag, p.err);
                __syncwarp();
                tc_fence_after();
                if (__any_sync(0xffffffffu, rescale)) {
                    const float a = rescale ? alpha : 1.f;
#pragma unroll
                    for (int cc = 0; cc < HD / 32; ++cc) {
                        float o[32];
                        tmem_ld32(tmem + lane_addr + C::O_COL + hf * HD + cc * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= a;
                        tmem_st32(tmem + lane_addr + C::O_COL + hf * HD + cc * 32, o);
                    }
                    tmem_wait_st();
                }
            }
            // P half-row -> shared memory (column block hf), 128B-swizzled K-major
#pragma unroll
            for (int ch = 0; ch < HC / 8; ++ch) {
                uint4 pk;
                if (kF16) {
                    __half2 h0 = __floats2half2_rn(s[ch * 8 + 0], s[ch * 8 + 1]);
                    __half2 h1 = __floats2half2_rn(s[ch * 8 + 2], s[ch * 8 + 3]);
                    __half2 h2 = __floats2half2_rn(s[ch * 8 + 4], s[ch * 8 + 5]);
                    __half2 h3 = __floats2half2_rn(s[ch * 8 + 6], s[ch * 8 + 7]);
                    pk.x = *reinterpret_cast<uint32_t *>(&h0);
                    pk.y = *reinterpret_cast<uint32_t *>(&h1);
                    pk.z = *reinterpret_cast<uint32_t *>(&h2);
                    pk.w = *reinterpret_cast<uint32_t *>(&h3);
                } else {
                    __nv_bfloat162 h0 = __floats2bfloat162_rn(s[ch * 8 + 0], s[ch * 8 + 1]);
                    __nv_bfloat162 h1 = __floats2bfloat162_rn(s[ch * 8 + 2], s[ch * 8 + 3]);
                    __nv_bfloat162 h2 = __floats2bfloat162_rn(s[ch * 8 + 4], s[ch * 8 + 5]);
                    __nv_bfloat162 h3 = __floats2bfloat162_rn(s[ch * 8 + 6], s[ch * 8 + 7]);
                    pk.x = *reinterpret_cast<uint32_t *>(&h0);
                    pk.y = *reinterpret_cast<uint32_t *>(&h1);
                    pk.z = *reinterpret_cast<uint32_t *>(&h2);
                    pk.w = *reinterpret_cast<uint32_t *>(&h3);
                }
                *reinterpret_cast<uint4 *>(prow + ((ch ^ (r & 7)) << 4)) = pk;
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }

        // epilogue: l = both halves' partial sums; O / l -> global
        xch[(4 + hf) * BM + r] = l_part;  // its own buffer: the partner may still read a max slot
        mbar_wait(o_done, (n_tiles - 1) & 1u, abort_flag, p.err);
        __syncwarp();
        named_bar_sync(2 + q4, 64);
        const float l_row = l_part + xch[(4 + (hf ^ 1u)) * BM + r];
        tc_fence_after();
        const float inv_l = 1.f / l_row;
        const bool valid = t < p.S;
        const size_t orow = ((size_t)(row_base + t) * p.H + h) * D + hf * HD;
#pragma unroll
        for (int cc = 0; cc < HD / 32; ++cc) {
            float o[32];
            tmem_ld32(tmem + lane_addr + C::O_COL + hf * HD + cc * 32, o);
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
                    for (int i = 0; i < 4; ++i) {
                        uint32_t w[4];
#pragma unroll
                        for (int k2 = 0; k2 < 4; ++k2) {
                            const float a0 = o[8 * i + 2 * k2] * inv_l, a1 = o[8 * i + 2 * k2 + 1] * inv_l;
                            if (kF16) {
                                __half2 hv = __floats2half2_rn(a0, a1);
                                w[k2] = *reinterpret_cast<uint32_t *>(&hv);
                            } else {
                                __nv_bfloat162 hv = __floats2bfloat162_rn(a0, a1);
                                w[k2] = *reinterpret_cast<uint32_t *>(&hv);
                            }
                        }
                        dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
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
    uint32_t *err = nullptr;
    cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_prefill_err);
    p.out = a.out;
    p.err = err;
    p.S = a.seq_len;
    p.H = a.n_heads;
    p.Hkv = a.n_kv;
    p.n_seqs = a.n_seqs;
    p.n_mtiles = (a.seq_len + BM - 1) / BM;
    p.scale_log2 = (float)((double)a.scale * 1.4426950408889634);
    p.causal = a.causal ? 1 : 0;
    p.out_f32 = a.out_dtype == BML_F32 ? 1 : 0;
    const uint64_t grid = (uint64_t)p.n_mtiles * a.n_seqs * a.n_heads;
    if (grid == 0 || grid > 0x7fffffffull) return cudaErrorInvalidValue;
    switch (a.head_dim) {
        case 64: return f16 ? launch_t<64, true>(p, (unsigned)grid, stream) : launch_t<64, false>(p, (unsigned)grid, stream);
        case 128:
            return f16 ? launch_t<128, true>(p, (unsigned)grid, stream) : launch_t<128, false>(p, (unsigned)grid, stream);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace bml
