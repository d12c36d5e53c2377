// decode_tc.cu -- split-K flash decoding on tcgen05 tensor cores (sm_100a),
// for 16-bit KV caches.
//
// Same result as decode.cu (the attention block of forward_layer_cached,
// crates/compiler/src/gguf_compiler.rs:1008-1050 in SugarFreeDoNoSo/bml,
// for every sequence of a batch), but the two contractions run on the
// tensor core so that the CUDA cores only do the softmax:
//
//   S^T[pos][n] = K[pos][:] . Qs[n][:]        M=128 positions, N=16/32, K=d
//   O^T[d][n]  += V[pos][d] . Ps[n][pos]      M=128 (d), N=16/32, K=128 pos
//
// Precision: q is f32.  It is written as the exact sum of three 16-bit
// terms q = q0 + q1 + q2 (q0 = round(q), q1 = round(q - q0), ...), which
// become three rows of Qs per q head; K is already 16-bit, every product of
// two 16-bit numbers is exact in f32, and the tensor core accumulates in
// f32, so S = sum of the three rows equals the f32 dot product to f32
// rounding.  P (f32) is split the same way into three rows of Ps.  Nothing
// is rounded to 16 bits that the reference keeps in 32 bits.
//
// Work: the units are (sequence, kv head); a tile is 128 consecutive
// positions of one unit.  A persistent grid of one CTA per SM walks a
// contiguous range of the flattened (unit, tile) list.  Warp roles:
//   warps 0-3  producers: 16-byte cp.async (L2 evict-first) of the K and V
//              rows of a tile into a 128B-swizzled 3-stage ring; rows past
//              the sequence end are zero-filled.
//   warps 4-7  softmax: thread r owns position r of the tile (TMEM lane r of
//              S^T) and, at the end of a unit, element d = r of O^T.
//   warp 8     allocates tensor memory; lane 0 issues every tcgen05.mma.
// Per tile the four softmax warps agree on one running max per q head
// (warp shuffles + one named barrier); O^T is rescaled in TMEM only when a
// max grows by more than 2^8.  A unit split over several CTAs leaves
// (m, l, o) partials in workspace slots; the last CTA of the unit (atomic
// ticket, reset afterwards) merges them in slot order.
#include <math.h>

#include "decode_tc.cuh"

namespace bml {

namespace {

constexpr int kTile = 128;
constexpr int kThreads = 288;  // 4 producer warps, 4 softmax warps, 1 MMA warp
constexpr float kRescaleThreshold = 8.0f;

template <int D, int N>
struct TcCfg {
    static constexpr int TILE_BYTES = kTile * D * 2;   // one K or V tile
    static constexpr int STAGES = D == 128 ? 3 : 4;
    static constexpr int P_BYTES = kTile * N * 2;     // one Ps buffer
    static constexpr int QS_BYTES = N * D * 2;
    // Layout: Ps buffers first, then Qs, then the ring, so that no operand
    // descriptor of this kernel can address past the allocation.
    static constexpr int OFF_P = 0;
    static constexpr int OFF_QS = OFF_P + 2 * P_BYTES;
    static constexpr int OFF_RING = ((OFF_QS + QS_BYTES + 1023) / 1024) * 1024;
    static constexpr int RING_BYTES = STAGES * 2 * TILE_BYTES;
    // With d=64 the O^T MMA still spans M=128 rows of V^T; the upper half
    // reads (and ignores) the 16 KiB after a V tile, which this pad keeps
    // inside the allocation.
    static constexpr int PAD = D == 64 ? 16384 : 0;
    static constexpr int OFF_BAR = OFF_RING + RING_BYTES + PAD;
    static constexpr int SMEM = OFF_BAR + 512 + 1024;
    static constexpr uint32_t TMEM_COLS = 128;
    static constexpr uint32_t S_COL = 0;        // two S^T buffers of N columns
    static constexpr uint32_t O_COL = 2 * N;    // O^T: N columns
};

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t src_bytes, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(smem_u32(dst)),
                 "l"(src), "r"(src_bytes), "l"(pol)
                 : "memory");
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float *v);

template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, float *v) {
    tmem_ld<16>(taddr, v);
    tmem_ld<16>(taddr + 16, v + 16);
}

template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const float *v);

template <>
__device__ __forceinline__ void tmem_st<16>(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
}

template <>
__device__ __forceinline__ void tmem_st<32>(uint32_t taddr, const float *v) {
    tmem_st<16>(taddr, v);
    tmem_st<16>(taddr + 16, v + 16);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (sm_100 version bit 46).  layout: 2 =
// 128-byte swizzle, 0 = no swizzle (8x16-byte core matrices).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// kind::f16 instruction descriptor, f32 accumulate.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t fmt, uint32_t m, uint32_t n, uint32_t a_mn, uint32_t b_mn) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Offset of 16-byte chunk c of row r in a 128B-swizzled K-major tile whose
// rows hold D 16-bit elements (D/64 column blocks of rows*128 bytes).
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c, uint32_t rows) {
    return (c >> 3) * (rows * 128u) + (r >> 3) * 1024u + (r & 7u) * 128u + (((c & 7u) ^ (r & 7u)) << 4);
}

template <bool F16>
__device__ __forceinline__ uint16_t to16(float x) {
    if (F16) return __half_as_ushort(__float2half_rn(x));
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
template <bool F16>
__device__ __forceinline__ float from16(uint16_t x) {
    if (F16) return __half2float(__ushort_as_half(x));
    return __bfloat162float(__ushort_as_bfloat16(x));
}

// x = t0 + t1 + t2 exactly (to f32 rounding of the remainders).
template <bool F16>
__device__ __forceinline__ void split3(float x, uint16_t &t0, uint16_t &t1, uint16_t &t2) {
    t0 = to16<F16>(x);
    const float r1 = x - from16<F16>(t0);
    t1 = to16<F16>(r1);
    const float r2 = r1 - from16<F16>(t1);
    t2 = to16<F16>(r2);
}

__device__ __forceinline__ uint32_t unit_tile_begin(const TcParams &p, uint32_t s, uint32_t h) {
    return p.seqs[s].tile_begin + h * p.seqs[s].tiles;
}

// ------------------------------------------------------------------ kernel
template <int D, int G, bool F16>
__global__ void __launch_bounds__(kThreads, 1) decode_tc_kernel(const __grid_constant__ TcParams p) {
    constexpr int N = G * 3 <= 16 ? 16 : 32;
    using C = TcCfg<D, N>;
    constexpr int KB = D / 64;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t *sP = smem + C::OFF_P;
    uint8_t *sQ = smem + C::OFF_QS;
    uint8_t *ring = smem + C::OFF_RING;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *kv_full = bars;               // [STAGES]
    uint64_t *kv_empty = kv_full + 4;       // [STAGES]
    uint64_t *s_full = kv_empty + 4;        // [2]
    uint64_t *s_empty = s_full + 2;         // [2]
    // P buffer b = i % 2 of tile i: p_full[b] when written, o_done[b] when
    // the P.V MMA that read it completed.  One barrier per buffer keeps every
    // waiter at most one phase behind its barrier.
    uint64_t *p_full = s_empty + 2;         // [2]
    uint64_t *o_done = p_full + 2;          // [2]
    uint64_t *q_ready = o_done + 2;
    volatile uint32_t *misc = reinterpret_cast<volatile uint32_t *>(q_ready + 1);  // [0] tmem [1] abort [2] last
    float *red = reinterpret_cast<float *>(smem + C::OFF_BAR + 256);             // [4][G] cross-warp values

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t t_begin = blockIdx.x * p.tiles_per_cta;
    const uint32_t t_end = min(t_begin + p.tiles_per_cta, p.total_tiles);

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::STAGES; ++i) {
            mbar_init(&kv_full[i], 128);
            mbar_init(&kv_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_empty[i], 4);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&p_full[i], 4);
            mbar_init(&o_done[i], 1);
        }
        mbar_init(q_ready, 4);
        misc[1] = 0u;
        misc[2] = 0u;
        fence_mbar_init();
    }
    if (warp == 8) {
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
    const bool has_work = t_begin < t_end;

    // unit and tile of global tile index t
    auto locate = [&](uint32_t t, uint32_t &s, uint32_t &h, uint32_t &j) {
        uint32_t ss = 0;
        while (ss + 1 < p.n_seqs && p.seqs[ss + 1].tile_begin <= t) ++ss;
        const uint32_t off = t - p.seqs[ss].tile_begin;
        s = ss;
        h = off / p.seqs[ss].tiles;
        j = off % p.seqs[ss].tiles;
    };

    if (has_work && warp < 4) {
        // ------------------------------------------------------- producers
        uint64_t pol;
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
        // Lanes cover whole rows so that every warp instruction reads
        // contiguous 128/256-byte row segments (full L2 sectors): lane l
        // copies 16-byte chunk (l % CPR) of row (l / CPR) of a group of RPI
        // rows; the four warps take every fourth group.
        constexpr int CPR = D / 8;           // 16-byte chunks per row of one head
        constexpr int RPI = 32 / CPR;        // rows per warp instruction
        const uint32_t c = lane % CPR, rsub = lane / CPR;
        uint32_t s, h, j;
        locate(t_begin, s, h, j);
        for (uint32_t t = t_begin, i = 0; t < t_end; ++t, ++i) {
            const uint32_t st = i % C::STAGES;
            if (i >= (uint32_t)C::STAGES) mbar_wait(&kv_empty[st], ((i / C::STAGES) & 1u) ^ 1u, abort_flag, p.err);
            __syncwarp();
            const TcSeq &sq = p.seqs[s];
            uint8_t *dk = ring + st * 2 * C::TILE_BYTES;
            uint8_t *dv = dk + C::TILE_BYTES;
            const uint8_t *kbase = static_cast<const uint8_t *>(sq.k) + (size_t)h * D * 2 + c * 16;
            const uint8_t *vbase = static_cast<const uint8_t *>(sq.v) + (size_t)h * D * 2 + c * 16;
#pragma unroll 4
            for (uint32_t g = warp; g < (uint32_t)(kTile / RPI); g += 4) {
                const uint32_t r = g * RPI + rsub;
                const uint32_t pos = j * kTile + r;
                const bool valid = pos < sq.len;
                const size_t off = valid ? (size_t)pos * p.row_bytes : 0;
                const uint32_t nb = valid ? 16u : 0u;
                const uint32_t o = swz(r, c, kTile);
                cp_async16(dk + o, kbase + off, nb, pol);
                cp_async16(dv + o, vbase + off, nb, pol);
            }
            cp_async_arrive_noinc(&kv_full[st]);
            if (++j == sq.tiles) {
                j = 0;
                if (++h == p.n_kv) {
                    h = 0;
                    ++s;
                }
            }
        }
    } else if (has_work && warp == 8) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t fmt = F16 ? 0u : 1u;
            constexpr uint32_t id_s = idesc_f16(fmt, 128, N, 0, 0);
            constexpr uint32_t id_o = idesc_f16(fmt, 128, N, 1, 1);
            const uint32_t ring_a = smem_u32(ring), q_a = smem_u32(sQ), p_a = smem_u32(sP);
            uint32_t s, h, j;
            locate(t_begin, s, h, j);
            uint32_t units = 0;  // units started (q_ready phases consumed)
            // S^T(i) for local tile i; returns after committing s_full
            auto issue_s = [&](uint32_t i, bool first_of_unit) {
                const uint32_t st = i % C::STAGES, sb = i & 1u;
                if (first_of_unit) {
                    mbar_wait(q_ready, units & 1u, abort_flag, p.err);
                    ++units;
                }
                mbar_wait(&kv_full[st], (i / C::STAGES) & 1u, abort_flag, p.err);
                if (i >= 2) mbar_wait(&s_empty[sb], ((i >> 1) & 1u) ^ 1u, abort_flag, p.err);
                fence_proxy_async_smem();
                tc_fence_after();
                const uint32_t k_a = ring_a + st * 2 * C::TILE_BYTES;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t ka = k_a + (kk >> 2) * (kTile * 128) + (kk & 3) * 32;
                    const uint32_t qa = q_a + (kk >> 2) * (N * 128) + (kk & 3) * 32;
                    tc_mma(tmem + C::S_COL + sb * N, sdesc(ka, 16, 1024, 2), sdesc(qa, 16, 1024, 2), id_s, kk > 0);
                }
                tc_commit(&s_full[sb]);
            };
            const uint32_t n = t_end - t_begin;
            // first-of-unit flags follow the tile walk
            uint32_t js = j;
            issue_s(0, true);
            bool first_next;
            for (uint32_t i = 0; i < n; ++i) {
                const bool first_this = (i == 0) || (js == 0);
                if (i + 1 < n) {
                    const uint32_t tiles_this = p.seqs[s].tiles;
                    first_next = (js + 1 == tiles_this);
                    issue_s(i + 1, first_next);
                }
                const uint32_t st = i % C::STAGES;
                mbar_wait(&p_full[i & 1u], (i >> 1) & 1u, abort_flag, p.err);
                tc_fence_after();
                const uint32_t v_a = ring_a + st * 2 * C::TILE_BYTES + C::TILE_BYTES;
                const uint32_t pb = p_a + (i & 1u) * C::P_BYTES;
#pragma unroll
                for (int kk = 0; kk < kTile / 16; ++kk) {
                    // A = V^T (MN-major, 128B swizzle): 16 positions = 2048 bytes
                    // B = Ps^T (MN-major, no swizzle): 16 positions x 16 bytes
                    tc_mma(tmem + C::O_COL, sdesc(v_a + kk * 2048, kTile * 128, 1024, 2),
                           sdesc(pb + kk * 256, 128, kTile * 16, 0), id_o, (!first_this || kk > 0) ? 1u : 0u);
                }
                tc_commit(&kv_empty[st]);
                tc_commit(&o_done[i & 1u]);
                // advance the unit walk
                if (++js == p.seqs[s].tiles) {
                    js = 0;
                    if (++h == p.n_kv) {
                        h = 0;
                        ++s;
                    }
                }
            }
            (void)j;
        }
        __syncwarp();
    } else if (has_work && warp >= 4 && warp < 8) {
        // ------------------------------------------------------- softmax
        const uint32_t w = warp - 4;              // == warp % 4: TMEM lane quarter
        const uint32_t r = w * 32 + lane;         // position within a tile / d of O^T
        const uint32_t lane_addr = (w * 32) << 16;
        const int tid = threadIdx.x - 128;        // 0..127
        constexpr int NB = N / 8;                 // 16-byte chunks of one Ps row
        uint32_t s, h, j;
        locate(t_begin, s, h, j);

        // Qs of unit (s, h): rows n = 3*g + k (k-th 16-bit term of q head g),
        // zero rows past 3G; 128B-swizzled K-major, N rows.
        auto build_q = [&](uint32_t ss, uint32_t hh) {
            const float *qg = p.q + ((size_t)ss * p.n_heads + (size_t)hh * G) * D;
            for (int idx = tid; idx < N * (D / 8); idx += 128) {
                const int row = idx / (D / 8), c = idx % (D / 8);
                uint16_t v[8];
                if (row < 3 * G) {
                    const int g = row / 3, k = row % 3;
                    const float4 *src = reinterpret_cast<const float4 *>(qg + (size_t)g * D + c * 8);
                    const float4 a = __ldg(src), b = __ldg(src + 1);
                    const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        uint16_t t0, t1, t2;
                        split3<F16>(x[e] * p.qscale, t0, t1, t2);
                        v[e] = k == 0 ? t0 : (k == 1 ? t1 : t2);
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = 0;
                }
                uint4 pk;
                pk.x = v[0] | ((uint32_t)v[1] << 16);
                pk.y = v[2] | ((uint32_t)v[3] << 16);
                pk.z = v[4] | ((uint32_t)v[5] << 16);
                pk.w = v[6] | ((uint32_t)v[7] << 16);
                *reinterpret_cast<uint4 *>(sQ + swz(row, c, N)) = pk;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_ready);  // 4 arrivals, one per warp
        };

        float m_run[G], l_part[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            m_run[g] = -INFINITY;
            l_part[g] = 0.f;
        }
        build_q(s, h);

        for (uint32_t t = t_begin, i = 0; t < t_end; ++t, ++i) {
            const TcSeq &sq = p.seqs[s];
            const bool last_of_unit = (j + 1 == sq.tiles) || (t + 1 == t_end);
            const bool first_of_unit = (j == 0) || (i == 0);
            const uint32_t sb = i & 1u;
            mbar_wait(&s_full[sb], (i >> 1) & 1u, abort_flag, p.err);
            __syncwarp();  // lanes leave the spin separately; tcgen05.ld needs the whole warp
            tc_fence_after();
            float sv[N];
            tmem_ld<N>(tmem + lane_addr + C::S_COL + sb * N, sv);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[sb]);

            // the next unit's Qs can be written as soon as this S^T is read
            uint32_t ns = s, nh = h;
            if (j + 1 == sq.tiles && t + 1 < t_end) {
                if (++nh == p.n_kv) {
                    nh = 0;
                    ++ns;
                }
                build_q(ns, nh);
            }

            // scores of this position for the G heads (log2 units)
            const uint32_t pos = j * kTile + r;
            const bool valid = pos < sq.len;
            float sc[G];
#pragma unroll
            for (int g = 0; g < G; ++g) sc[g] = valid ? (sv[3 * g] + sv[3 * g + 1]) + sv[3 * g + 2] : -INFINITY;
            // tile max per head across the 128 positions
            float mx[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float v = sc[g];
#pragma unroll
                for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
                mx[g] = v;
            }
            if (lane == 0) {
#pragma unroll
                for (int g = 0; g < G; ++g) red[w * G + g] = mx[g];
            }
            __syncwarp();
            named_bar_sync(2, 128);
            float alpha[G];
            bool rescale = false;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float mt = fmaxf(fmaxf(red[g], red[G + g]), fmaxf(red[2 * G + g], red[3 * G + g]));
                float mn = m_run[g];
                if (m_run[g] == -INFINITY || mt > m_run[g] + kRescaleThreshold) mn = fmaxf(m_run[g], mt);
                alpha[g] = (m_run[g] == -INFINITY || mn == -INFINITY) ? 1.f : fast_exp2(m_run[g] - mn);
                rescale |= (!first_of_unit && mn != m_run[g]);
                m_run[g] = mn;
            }
            __syncwarp();
            named_bar_sync(2, 128);  // red[] is rewritten next tile
            float pv[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float mu = m_run[g] == -INFINITY ? 0.f : m_run[g];
                pv[g] = (sc[g] == -INFINITY) ? 0.f : fast_exp2(sc[g] - mu);
                l_part[g] = first_of_unit ? pv[g] : l_part[g] * alpha[g] + pv[g];
            }
            // O^T rescale (rare): all 128 threads own one d each
            if (rescale) {
                mbar_wait(&o_done[(i - 1) & 1u], ((i - 1) >> 1) & 1u, abort_flag, p.err);
                __syncwarp();
                tc_fence_after();
                float o[N];
                tmem_ld<N>(tmem + lane_addr + C::O_COL, o);
                tmem_wait_ld();
#pragma unroll
                for (int n2 = 0; n2 < N; ++n2) o[n2] *= (n2 < 3 * G) ? alpha[n2 / 3] : 1.f;
                tmem_st<N>(tmem + lane_addr + C::O_COL, o);
                tmem_wait_st();
            }
            // Ps^T row of this position: 3 terms per head, zero padding
            if (i >= 2) mbar_wait(&o_done[sb], ((i - 2) >> 1) & 1u, abort_flag, p.err);  // PV(i-2) freed it
            __syncwarp();
            uint16_t terms[N];
#pragma unroll
            for (int n2 = 0; n2 < N; ++n2) terms[n2] = 0;
#pragma unroll
            for (int g = 0; g < G; ++g) split3<F16>(pv[g], terms[3 * g], terms[3 * g + 1], terms[3 * g + 2]);
            uint8_t *pb = sP + sb * C::P_BYTES + r * 16;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                uint4 pk;
                pk.x = terms[8 * b + 0] | ((uint32_t)terms[8 * b + 1] << 16);
                pk.y = terms[8 * b + 2] | ((uint32_t)terms[8 * b + 3] << 16);
                pk.z = terms[8 * b + 4] | ((uint32_t)terms[8 * b + 5] << 16);
                pk.w = terms[8 * b + 6] | ((uint32_t)terms[8 * b + 7] << 16);
                *reinterpret_cast<uint4 *>(pb + b * (kTile * 16)) = pk;
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[sb]);

            if (last_of_unit) {
                // ------------------------------------------- finalize unit (s, h)
                mbar_wait(&o_done[sb], (i >> 1) & 1u, abort_flag, p.err);
                __syncwarp();
                tc_fence_after();
                float lsum[G];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float v = l_part[g];
#pragma unroll
                    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
                    lsum[g] = v;
                }
                if (lane == 0) {
#pragma unroll
                    for (int g = 0; g < G; ++g) red[w * G + g] = lsum[g];
                }
                __syncwarp();
            named_bar_sync(2, 128);
                float L[G];
#pragma unroll
                for (int g = 0; g < G; ++g) L[g] = (red[g] + red[G + g]) + (red[2 * G + g] + red[3 * G + g]);
                __syncwarp();
            named_bar_sync(2, 128);
                float o[N];
                tmem_ld<N>(tmem + lane_addr + C::O_COL, o);
                tmem_wait_ld();
                const uint32_t d = r;
                const uint32_t unit = s * p.n_kv + h;
                const uint32_t ub = unit_tile_begin(p, s, h);
                const uint32_t first_cta = ub / p.tiles_per_cta;
                const uint32_t last_cta = (ub + sq.tiles - 1) / p.tiles_per_cta;
                const uint32_t n_slots = last_cta - first_cta + 1;
                if (d < (uint32_t)D) {
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float og = ((o[3 * g] + o[3 * g + 1]) + o[3 * g + 2]) / L[g];
                        const size_t row = (size_t)s * p.n_heads + (size_t)h * G + g;
                        if (n_slots == 1) {
                            if (p.mode == kModeFinal) {
                                p.out[row * D + d] = og;
                            } else {
                                p.part_o[row * D + d] = og;
                                if (d == 0) {
                                    p.part_m[row] = m_run[g];
                                    p.part_l[row] = L[g];
                                }
                            }
                        } else {
                            const size_t slot = (size_t)sq.slot_base + (size_t)h * sq.slots_per_unit +
                                                (blockIdx.x - first_cta);
                            p.slot_o[(slot * G + g) * D + d] = og;
                            if (d == 0) {
                                p.slot_ml[(slot * G + g) * 2] = m_run[g];
                                p.slot_ml[(slot * G + g) * 2 + 1] = L[g];
                            }
                        }
                    }
                }
                if (n_slots > 1) {
                    __threadfence();
                    __syncwarp();
            named_bar_sync(2, 128);
                    if (tid == 0) {
                        const uint32_t old = atomicAdd(&p.counters[unit], 1u);
                        misc[2] = (old == n_slots - 1) ? 1u : 0u;
                    }
                    __syncwarp();
            named_bar_sync(2, 128);
                    if (misc[2]) {
                        __threadfence();
                        const size_t base = (size_t)sq.slot_base + (size_t)h * sq.slots_per_unit;
                        for (int idx = tid; idx < G * D; idx += 128) {
                            const int g = idx / D, dd = idx % D;
                            float M = -INFINITY;
                            for (uint32_t k = 0; k < n_slots; ++k)
                                M = fmaxf(M, __ldcg(&p.slot_ml[((base + k) * G + g) * 2]));
                            float Ls = 0.f, O = 0.f;
                            for (uint32_t k = 0; k < n_slots; ++k) {
                                const float mk = __ldcg(&p.slot_ml[((base + k) * G + g) * 2]);
                                const float f = (mk == -INFINITY) ? 0.f
                                                                  : fast_exp2(mk - M) * __ldcg(&p.slot_ml[((base + k) * G + g) * 2 + 1]);
                                Ls += f;
                                O += __ldcg(&p.slot_o[((base + k) * G + g) * D + dd]) * f;
                            }
                            const size_t row = (size_t)s * p.n_heads + (size_t)h * G + g;
                            if (p.mode == kModeFinal) {
                                p.out[row * D + dd] = O / Ls;
                            } else {
                                p.part_o[row * D + dd] = O / Ls;
                                if (dd == 0) {
                                    p.part_m[row] = M;
                                    p.part_l[row] = Ls;
                                }
                            }
                        }
                        if (tid == 0) p.counters[unit] = 0u;
                    }
                    __syncwarp();
            named_bar_sync(2, 128);
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    m_run[g] = -INFINITY;
                    l_part[g] = 0.f;
                }
            }
            // advance the unit walk
            if (++j == sq.tiles) {
                j = 0;
                if (++h == p.n_kv) {
                    h = 0;
                    ++s;
                }
            }
        }
        tc_fence_before();
    }

    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS)
                     : "memory");
    }
}

template <int D, int G, bool F16>
cudaError_t launch_t(const TcParams &p, int grid, cudaStream_t stream) {
    constexpr int N = G * 3 <= 16 ? 16 : 32;
    constexpr int smem = TcCfg<D, N>::SMEM;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_tc_kernel<D, G, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    decode_tc_kernel<D, G, F16><<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

template <int D, bool F16>
cudaError_t launch_g(const TcParams &p, uint32_t group, int grid, cudaStream_t stream) {
    switch (group) {
        case 1: return launch_t<D, 1, F16>(p, grid, stream);
        case 2: return launch_t<D, 2, F16>(p, grid, stream);
        case 4: return launch_t<D, 4, F16>(p, grid, stream);
        case 8: return launch_t<D, 8, F16>(p, grid, stream);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace

bool decode_tc_supported(bml_dtype dt, uint32_t head_dim, uint32_t group) {
    return (dt == BML_BF16 || dt == BML_F16) && (head_dim == 64 || head_dim == 128) &&
           (group == 1 || group == 2 || group == 4 || group == 8);
}

cudaError_t launch_decode_tc(const TcParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group, int grid,
                             cudaStream_t stream) {
    const bool f16 = dt == BML_F16;
    if (head_dim == 128) return f16 ? launch_g<128, true>(p, group, grid, stream) : launch_g<128, false>(p, group, grid, stream);
    if (head_dim == 64) return f16 ? launch_g<64, true>(p, group, grid, stream) : launch_g<64, false>(p, group, grid, stream);
    return cudaErrorNotSupported;
}

}  // namespace bml
