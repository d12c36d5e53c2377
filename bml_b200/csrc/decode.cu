// decode.cu -- split-K flash decoding over per-sequence KV caches (sm_100a).
//
// Computes, for every sequence of a batch, the attention block of
// forward_layer_cached (crates/compiler/src/gguf_compiler.rs:1008-1050 in
// SugarFreeDoNoSo/bml): scores q.k * scale over every cached position, a
// max-subtracted softmax and the P.V sum, for the n_heads/n_kv q heads that
// share each kv head.  q stays f32 and every product and sum is f32, so the
// result matches the reference's f32/f64 arithmetic to ~1e-6.
//
// Design (HBM-bound: each K/V byte is read exactly once):
//  * Persistent grid: one CTA per SM walks a contiguous range of the
//    flattened list of (sequence, tile) work, so ragged batches balance to
//    within one tile per SM.  A tile is T consecutive positions of ALL kv
//    heads, which is one contiguous run of T*n_kv*D elements.
//  * Thread 0 streams tiles into a 4-stage shared-memory ring with 1-D TMA
//    bulk copies (cp.async.bulk, L2 evict-first) completing on mbarriers;
//    the 8 warps release stages through a second mbarrier ring and thread 0
//    refills a stage once all of them have released it.
//  * 8 consumer warps: warp w serves kv head w % n_kv.  Inside a warp, 8
//    lanes share one KV row (16-byte conflict-free shared loads), so a warp
//    covers 4 rows per step.  q for the G heads of the group stays in
//    registers, pre-scaled by scale*log2(e).
//  * Per tile: pass 1 computes the G dot products of each row and reduces
//    them across the 8 lanes with a transposing butterfly (lane j ends up
//    owning head j*G/8, so each (row, head) exponent is computed once);
//    running max / sum per (lane group, head); pass 2 accumulates P.V.
//  * A CTA's partial for a sequence is merged across lane groups (shuffles)
//    and warps (shared memory).  A sequence handled by one CTA is written
//    directly; otherwise partials (m, l, o) go to workspace slots and the
//    last CTA to finish that sequence (atomic ticket, reset afterwards)
//    merges them with the log-sum-exp rule in slot order.
#include <math.h>

#include "decode.cuh"

namespace bml {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads;
constexpr int kSmemBudget = 227 * 1024;

template <typename KT, int D, int G>
struct Cfg {
    static constexpr int ES = sizeof(KT);
    static constexpr int HEAD_BYTES = D * ES;
    static constexpr int CHUNKS = HEAD_BYTES / 16;
    static constexpr int CPL = CHUNKS / 8;  // 16-byte chunks per lane
    static constexpr int EPC = 16 / ES;     // elements per chunk
    static constexpr int E = CPL * EPC;     // elements per lane
    static constexpr int E2 = E / 2;        // float2 pairs per lane
    static constexpr int STAGE_K = 32768;   // K bytes per stage; V the same
    // rows per warp per step = 4; stage bytes = STEPS * 4 rows * 8 warps * HEAD_BYTES
    static constexpr int STEPS = STAGE_K / (32 * HEAD_BYTES);
    static constexpr int WSCR = 4 * G /*alpha*/ + 4 * STEPS * G /*p*/ + 4 * G * 2 /*ml*/;
    static constexpr int EXTRA = 2 * 8 * 8 /*barriers*/ + 16 +
                                 4 * (kConsumerWarps * WSCR + kConsumerWarps * G * D + kConsumerWarps * G * 2);
    static constexpr int STAGES_FIT = (kSmemBudget - EXTRA) / (2 * STAGE_K);
    static constexpr int STAGES = STAGES_FIT > 4 ? 4 : STAGES_FIT;
    static constexpr int BAR_OFF = STAGES * 2 * STAGE_K;
    static constexpr int SMEM = BAR_OFF + EXTRA;
    static_assert(CHUNKS % 8 == 0, "head row must be a multiple of 128 bytes");
    static_assert(STEPS >= 1, "stage too small");
    static_assert(STAGES >= 2, "shared memory budget");
};

__device__ __forceinline__ uint32_t seq_of_tile(const DecodeParams &p, uint32_t t) {
    uint32_t s = 0;
    while (s + 1 < p.n_seqs && p.seqs[s + 1].tile_begin <= t) ++s;
    return s;
}

__device__ __forceinline__ uint32_t tile_end_of(const DecodeParams &p, uint32_t s) {
    return s + 1 < p.n_seqs ? p.seqs[s + 1].tile_begin : p.total_tiles;
}

// Butterfly reduction of G per-lane partial sums across the 8 lanes of a
// lane group that also transposes: on return, lane j (j = lane & 7) holds
// the full sum of value index j*G/8.
template <int G>
__device__ __forceinline__ float transpose_reduce(float (&v)[G], int j) {
    constexpr unsigned FULL = 0xffffffffu;
    int n = G;
#pragma unroll
    for (int lvl = 0; lvl < 3; ++lvl) {
        const int mask = 4 >> lvl;
        const bool upper = (j & mask) != 0;
        if (n >= 2) {
            const int half = n / 2;
#pragma unroll
            for (int i = 0; i < G / 2; ++i) {
                if (i < half) {
                    const float send = upper ? v[i] : v[i + half];
                    const float keep = upper ? v[i + half] : v[i];
                    v[i] = keep + __shfl_xor_sync(FULL, send, mask);
                }
            }
            n = half;
        } else {
            v[0] += __shfl_xor_sync(FULL, v[0], mask);
        }
    }
    return v[0];
}

template <typename KT, int D, int G>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    using C = Cfg<KT, D, G>;
    constexpr int STEPS = C::STEPS, E2 = C::E2, CPL = C::CPL, EPC = C::EPC;
    constexpr int HEAD_BYTES = C::HEAD_BYTES, STAGE_K = C::STAGE_K, NST = C::STAGES;
    constexpr int WSCR = C::WSCR;
    constexpr float NEG_INF = -INFINITY;

    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *stages = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *empty = full + 8;
    volatile uint32_t *flags = reinterpret_cast<volatile uint32_t *>(empty + 8);
    float *wscr = reinterpret_cast<float *>(smem + C::BAR_OFF + 2 * 8 * 8 + 16);
    float *wsum = wscr + kConsumerWarps * WSCR;  // [8 warps][G][D]
    float *wml = wsum + kConsumerWarps * G * D;  // [8 warps][G][2]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t t_begin = blockIdx.x * p.tiles_per_cta;
    const uint32_t t_end = min(t_begin + p.tiles_per_cta, p.total_tiles);
    const uint32_t T = p.rows_per_tile;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        flags[0] = 0u;
        flags[1] = 0u;
        fence_mbar_init();
    }
    __syncthreads();
    if (t_begin >= t_end) return;

    // Thread 0 doubles as the producer: it fills the ring ahead of the
    // consumers and refills a stage as soon as all 8 warps released it.
    // (A separate producer warp would make 9 warps; the register file is
    // split over 4 sub-partitions, and a 3-warp partition caps a thread at
    // 168 registers, below what the consumers need.)
    uint64_t pol = 0;
    uint32_t ps = 0, pt = t_begin;  // producer cursor: sequence, tile
    auto issue = [&](uint32_t it) {
        while (pt >= tile_end_of(p, ps)) ++ps;
        const uint32_t stage = it % NST;
        const uint32_t row0 = (pt - p.seqs[ps].tile_begin) * T;
        const uint32_t rows = min(T, p.seqs[ps].len - row0);
        const uint32_t bytes = rows * p.row_bytes;
        uint8_t *sk = stages + stage * 2 * STAGE_K;
        mbar_arrive_expect_tx(&full[stage], 2 * bytes);
        const uint8_t *gk = static_cast<const uint8_t *>(p.seqs[ps].k) + (size_t)row0 * p.row_bytes;
        const uint8_t *gv = static_cast<const uint8_t *>(p.seqs[ps].v) + (size_t)row0 * p.row_bytes;
        bulk_g2s_stream(sk, gk, bytes, &full[stage], pol);
        bulk_g2s_stream(sk + STAGE_K, gv, bytes, &full[stage], pol);
        ++pt;
    };
    const uint32_t n_tiles = t_end - t_begin;
    if (threadIdx.x == 0) {
        pol = l2_policy_evict_first();
        ps = seq_of_tile(p, t_begin);
        for (uint32_t it = 0; it < n_tiles && it < (uint32_t)NST; ++it) issue(it);
    }

    const int n_kv = (int)p.n_kv;
    const int nwh = kConsumerWarps / n_kv;  // warps per kv head
    const int h = warp % n_kv, ph = warp / n_kv;
    const int grp = lane >> 3, j = lane & 7;
    const int own = (j * G) >> 3;
    const bool owner_lane = (j & ((8 / G) - 1)) == 0;
    float *scr = wscr + warp * WSCR;
    float *s_alpha = scr;               // [4][G]
    float *s_p = scr + 4 * G;           // [4][STEPS][G]
    float *s_ml = s_p + 4 * STEPS * G;  // [4][G][2]

    float2 q2[G][E2], acc[G][E2];
    float m_own = NEG_INF, l_own = 0.f;

    uint32_t s = seq_of_tile(p, t_begin);
    auto load_q = [&](uint32_t seq) {
        const float *qs = p.q + ((size_t)seq * p.n_heads + (size_t)h * G) * D;
#pragma unroll
        for (int hh = 0; hh < G; ++hh) {
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                const float4 *src = reinterpret_cast<const float4 *>(qs + hh * D + (j + 8 * c) * EPC);
#pragma unroll
                for (int f = 0; f < EPC / 4; ++f) {
                    const float4 v = __ldg(src + f);
                    q2[hh][(c * EPC) / 2 + 2 * f + 0] = make_float2(v.x * p.qscale, v.y * p.qscale);
                    q2[hh][(c * EPC) / 2 + 2 * f + 1] = make_float2(v.z * p.qscale, v.w * p.qscale);
                }
            }
        }
#pragma unroll
        for (int hh = 0; hh < G; ++hh)
#pragma unroll
            for (int e = 0; e < E2; ++e) acc[hh][e] = make_float2(0.f, 0.f);
        m_own = NEG_INF;
        l_own = 0.f;
    };
    load_q(s);

    for (uint32_t t = t_begin, it = 0; t < t_end; ++t, ++it) {
        const uint32_t stage = it % NST;
        mbar_wait(&full[stage], (it / NST) & 1u, flags, p.err);
        const uint32_t row0 = (t - p.seqs[s].tile_begin) * T;
        const uint32_t rows = min(T, p.seqs[s].len - row0);
        const uint8_t *sk = stages + stage * 2 * STAGE_K + h * HEAD_BYTES;
        const uint8_t *sv = sk + STAGE_K;

        // pass 1: scores of this lane group's rows (log2 domain)
        float sc[STEPS];
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
            const uint32_t r = (uint32_t)((st * nwh + ph) * 4 + grp);
            float2 part2[G];
#pragma unroll
            for (int hh = 0; hh < G; ++hh) part2[hh] = make_float2(0.f, 0.f);
            if (r < rows) {
                const uint8_t *rowp = sk + (size_t)r * p.row_bytes;
#pragma unroll
                for (int c = 0; c < CPL; ++c) {
                    const uint4 raw = *reinterpret_cast<const uint4 *>(rowp + (j + 8 * c) * 16);
                    float2 kf[EPC / 2];
                    Elem<KT>::widen2(raw, kf);
#pragma unroll
                    for (int hh = 0; hh < G; ++hh)
#pragma unroll
                        for (int e = 0; e < EPC / 2; ++e)
                            part2[hh] = __ffma2_rn(q2[hh][c * (EPC / 2) + e], kf[e], part2[hh]);
                }
            }
            float part[G];
#pragma unroll
            for (int hh = 0; hh < G; ++hh) part[hh] = part2[hh].x + part2[hh].y;
            const float tot = transpose_reduce<G>(part, j);
            sc[st] = (r < rows) ? tot : NEG_INF;
        }
        float mt = sc[0];
#pragma unroll
        for (int st = 1; st < STEPS; ++st) mt = fmaxf(mt, sc[st]);
        const float m_new = fmaxf(m_own, mt);
        const float alpha = (m_new == NEG_INF) ? 1.f : fast_exp2(m_own - m_new);
        float psum = 0.f;
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
            const float pv = (sc[st] == NEG_INF) ? 0.f : fast_exp2(sc[st] - m_new);
            sc[st] = pv;
            psum += pv;
        }
        l_own = l_own * alpha + psum;
        m_own = m_new;
        if (owner_lane) {
            s_alpha[grp * G + own] = alpha;
#pragma unroll
            for (int st = 0; st < STEPS; ++st) s_p[(grp * STEPS + st) * G + own] = sc[st];
        }
        __syncwarp();

        // rescale the accumulators when a running max moved
        float al[G];
        bool moved = false;
#pragma unroll
        for (int hh = 0; hh < G; ++hh) {
            al[hh] = s_alpha[grp * G + hh];
            moved |= (al[hh] != 1.f);
        }
        if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
            for (int hh = 0; hh < G; ++hh) {
                const float2 a2 = make_float2(al[hh], al[hh]);
#pragma unroll
                for (int e = 0; e < E2; ++e) acc[hh][e] = __fmul2_rn(acc[hh][e], a2);
            }
        }

        // pass 2: P.V
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
            const uint32_t r = (uint32_t)((st * nwh + ph) * 4 + grp);
            if (r < rows) {
                float2 pp[G];
#pragma unroll
                for (int hh = 0; hh < G; ++hh) {
                    const float pv = s_p[(grp * STEPS + st) * G + hh];
                    pp[hh] = make_float2(pv, pv);
                }
                const uint8_t *rowp = sv + (size_t)r * p.row_bytes;
#pragma unroll
                for (int c = 0; c < CPL; ++c) {
                    const uint4 raw = *reinterpret_cast<const uint4 *>(rowp + (j + 8 * c) * 16);
                    float2 vf[EPC / 2];
                    Elem<KT>::widen2(raw, vf);
#pragma unroll
                    for (int hh = 0; hh < G; ++hh)
#pragma unroll
                        for (int e = 0; e < EPC / 2; ++e)
                            acc[hh][c * (EPC / 2) + e] = __ffma2_rn(pp[hh], vf[e], acc[hh][c * (EPC / 2) + e]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (threadIdx.x == 0 && it + NST < n_tiles) {
            mbar_wait(&empty[stage], (it / NST) & 1u, flags, p.err);
            issue(it + NST);
        }

        const bool last_of_cta = (t + 1 == t_end);
        const bool seq_done = (t + 1 == tile_end_of(p, s));
        if (!(last_of_cta || seq_done)) continue;

        // ---------------------------------------------- finalize sequence s
        if (owner_lane) {
            s_ml[(grp * G + own) * 2 + 0] = m_own;
            s_ml[(grp * G + own) * 2 + 1] = l_own;
        }
        __syncwarp();
        float Mh[G], Lh[G];
#pragma unroll
        for (int hh = 0; hh < G; ++hh) {
            float mg[4], lg[4];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                mg[g] = s_ml[(g * G + hh) * 2 + 0];
                lg[g] = s_ml[(g * G + hh) * 2 + 1];
            }
            const float M = fmaxf(fmaxf(mg[0], mg[1]), fmaxf(mg[2], mg[3]));
            float L = 0.f, mine = 0.f;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const float f = (mg[g] == NEG_INF) ? 0.f : fast_exp2(mg[g] - M);
                L += lg[g] * f;
                if (g == grp) mine = f;
            }
            Mh[hh] = M;
            Lh[hh] = L;
            const float2 f2 = make_float2(mine, mine);
#pragma unroll
            for (int e = 0; e < E2; ++e) acc[hh][e] = __fmul2_rn(acc[hh][e], f2);
        }
#pragma unroll
        for (int hh = 0; hh < G; ++hh)
#pragma unroll
            for (int e = 0; e < E2; ++e) {
                acc[hh][e].x += __shfl_xor_sync(0xffffffffu, acc[hh][e].x, 8);
                acc[hh][e].y += __shfl_xor_sync(0xffffffffu, acc[hh][e].y, 8);
                acc[hh][e].x += __shfl_xor_sync(0xffffffffu, acc[hh][e].x, 16);
                acc[hh][e].y += __shfl_xor_sync(0xffffffffu, acc[hh][e].y, 16);
            }
        float *ws = wsum + warp * G * D;
        if (grp == 0) {
#pragma unroll
            for (int hh = 0; hh < G; ++hh)
#pragma unroll
                for (int c = 0; c < CPL; ++c)
#pragma unroll
                    for (int e = 0; e < EPC / 2; ++e)
                        *reinterpret_cast<float2 *>(ws + hh * D + (j + 8 * c) * EPC + 2 * e) = acc[hh][c * (EPC / 2) + e];
        }
        if (lane == 0) {
#pragma unroll
            for (int hh = 0; hh < G; ++hh) {
                wml[(warp * G + hh) * 2 + 0] = Mh[hh];
                wml[(warp * G + hh) * 2 + 1] = Lh[hh];
            }
        }
        named_bar_sync(1, kConsumerThreads);

        const DecodeSeq &sq = p.seqs[s];
        const bool single = (sq.n_slots == 1);
        const uint32_t slot = sq.slot_base + (blockIdx.x - sq.tile_begin / p.tiles_per_cta);
        const uint32_t total = p.n_heads * D;
        const int tid = threadIdx.x;
        for (uint32_t idx = tid; idx < total; idx += kConsumerThreads) {
            const uint32_t qh = idx / D, d = idx % D;
            const uint32_t hk = qh / G, hh = qh % G;
            float M = NEG_INF;
            for (int w = 0; w < nwh; ++w) M = fmaxf(M, wml[((hk + w * n_kv) * G + hh) * 2]);
            float L = 0.f, O = 0.f;
            for (int w = 0; w < nwh; ++w) {
                const int ww = hk + w * n_kv;
                const float mw = wml[(ww * G + hh) * 2];
                const float f = (mw == NEG_INF) ? 0.f : fast_exp2(mw - M);
                L += wml[(ww * G + hh) * 2 + 1] * f;
                O += wsum[(ww * G + hh) * D + d] * f;
            }
            const float o = O / L;
            const size_t row = (size_t)s * p.n_heads + qh;
            if (single) {
                if (p.mode == kModeFinal) {
                    p.out[row * D + d] = o;
                } else {
                    p.part_o[row * D + d] = o;
                    if (d == 0) {
                        p.part_m[row] = M;
                        p.part_l[row] = L;
                    }
                }
            } else {
                p.slot_o[((size_t)slot * p.n_heads + qh) * D + d] = o;
                if (d == 0) {
                    p.slot_ml[((size_t)slot * p.n_heads + qh) * 2 + 0] = M;
                    p.slot_ml[((size_t)slot * p.n_heads + qh) * 2 + 1] = L;
                }
            }
        }
        if (!single) {
            __threadfence();
            named_bar_sync(1, kConsumerThreads);
            if (tid == 0) {
                const uint32_t old = atomicAdd(&p.counters[s], 1u);
                flags[1] = (old == sq.n_slots - 1) ? 1u : 0u;
            }
            named_bar_sync(1, kConsumerThreads);
            if (flags[1]) {
                __threadfence();
                for (uint32_t idx = tid; idx < total; idx += kConsumerThreads) {
                    const uint32_t qh = idx / D, d = idx % D;
                    float M = NEG_INF;
                    for (uint32_t i = 0; i < sq.n_slots; ++i)
                        M = fmaxf(M, __ldcg(&p.slot_ml[((size_t)(sq.slot_base + i) * p.n_heads + qh) * 2]));
                    float L = 0.f, O = 0.f;
                    for (uint32_t i = 0; i < sq.n_slots; ++i) {
                        const size_t sr = (size_t)(sq.slot_base + i) * p.n_heads + qh;
                        const float mi = __ldcg(&p.slot_ml[sr * 2]);
                        const float li = __ldcg(&p.slot_ml[sr * 2 + 1]);
                        const float f = (mi == NEG_INF) ? 0.f : fast_exp2(mi - M) * li;
                        L += f;
                        O += __ldcg(&p.slot_o[sr * D + d]) * f;
                    }
                    const size_t row = (size_t)s * p.n_heads + qh;
                    if (p.mode == kModeFinal) {
                        p.out[row * D + d] = O / L;
                    } else {
                        p.part_o[row * D + d] = O / L;
                        if (d == 0) {
                            p.part_m[row] = M;
                            p.part_l[row] = L;
                        }
                    }
                }
                if (tid == 0) p.counters[s] = 0u;
            }
        }
        named_bar_sync(1, kConsumerThreads);
        if (!last_of_cta) {
            ++s;
            load_q(s);
        }
    }
}

template <typename KT, int D, int G>
cudaError_t launch_one(const DecodeParams &p, int grid, cudaStream_t stream) {
    constexpr int smem = Cfg<KT, D, G>::SMEM;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<KT, D, G>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    decode_kernel<KT, D, G><<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

template <typename KT, int D>
cudaError_t launch_g(const DecodeParams &p, uint32_t group, int grid, cudaStream_t stream) {
    switch (group) {
        case 1: return launch_one<KT, D, 1>(p, grid, stream);
        case 2: return launch_one<KT, D, 2>(p, grid, stream);
        case 4: return launch_one<KT, D, 4>(p, grid, stream);
        case 8: return launch_one<KT, D, 8>(p, grid, stream);
        default: return cudaErrorNotSupported;
    }
}

template <typename KT>
cudaError_t launch_d(const DecodeParams &p, uint32_t head_dim, uint32_t group, int grid,
                     cudaStream_t stream) {
    switch (head_dim) {
        case 64: return launch_g<KT, 64>(p, group, grid, stream);
        case 128: return launch_g<KT, 128>(p, group, grid, stream);
        default: return cudaErrorNotSupported;
    }
}

__global__ void merge_lse_kernel(const float *__restrict__ m, const float *__restrict__ l,
                                 const float *__restrict__ o, uint32_t n_parts, uint32_t n_rows,
                                 uint32_t head_dim, float *__restrict__ out) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t total = (size_t)n_rows * head_dim;
    if (idx >= total) return;
    const size_t row = idx / head_dim, d = idx % head_dim;
    float M = -INFINITY;
    for (uint32_t i = 0; i < n_parts; ++i) M = fmaxf(M, m[(size_t)i * n_rows + row]);
    float L = 0.f, O = 0.f;
    for (uint32_t i = 0; i < n_parts; ++i) {
        const float mi = m[(size_t)i * n_rows + row];
        const float f = (mi == -INFINITY) ? 0.f : fast_exp2(mi - M) * l[(size_t)i * n_rows + row];
        L += f;
        O += o[((size_t)i * n_rows + row) * head_dim + d] * f;
    }
    out[idx] = O / L;
}

// Packed parts: part i holds m [n_rows] | l [n_rows] | o [n_rows][d].
__global__ void merge_lse_packed_kernel(const float *__restrict__ parts, uint32_t n_parts,
                                        uint32_t n_rows, uint32_t head_dim, float *__restrict__ out) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t total = (size_t)n_rows * head_dim;
    if (idx >= total) return;
    const size_t row = idx / head_dim, d = idx % head_dim;
    const size_t part = (size_t)n_rows * (head_dim + 2);
    float M = -INFINITY;
    for (uint32_t i = 0; i < n_parts; ++i) M = fmaxf(M, parts[i * part + row]);
    float L = 0.f, O = 0.f;
    for (uint32_t i = 0; i < n_parts; ++i) {
        const float *p = parts + i * part;
        const float mi = p[row];
        const float f = (mi == -INFINITY) ? 0.f : fast_exp2(mi - M) * p[n_rows + row];
        L += f;
        O += p[2 * (size_t)n_rows + row * head_dim + d] * f;
    }
    out[idx] = O / L;
}

}  // namespace

uint32_t decode_rows_per_tile(bml_dtype dt, uint32_t head_dim, uint32_t n_kv) {
    // STEPS * 4 rows * (8 / n_kv) warps per head; equal to STAGE_K / row_bytes
    const uint32_t row_bytes = n_kv * head_dim * (uint32_t)dtype_size(dt);
    return 32768u / row_bytes;
}

size_t decode_workspace_bytes(uint32_t n_seqs, uint32_t n_heads, uint32_t head_dim, int num_sms) {
    const size_t seqs = n_seqs < (uint32_t)kMaxSeqsPerLaunch ? n_seqs : kMaxSeqsPerLaunch;
    const size_t slots = seqs + (size_t)num_sms;
    size_t b = 256;                                     // error word
    b += ((seqs * 4 + 255) / 256) * 256;                // counters
    b += ((slots * n_heads * 2 * 4 + 255) / 256) * 256; // slot (m, l)
    b += slots * n_heads * head_dim * 4;                // slot o
    return b;
}

bool decode_workspace_carve(void *ws, size_t bytes, uint32_t n_seqs, uint32_t n_heads,
                            uint32_t head_dim, int num_sms, DecodeWorkspace *out) {
    if (!ws || bytes < decode_workspace_bytes(n_seqs, n_heads, head_dim, num_sms)) return false;
    const size_t seqs = n_seqs < (uint32_t)kMaxSeqsPerLaunch ? n_seqs : kMaxSeqsPerLaunch;
    const size_t slots = seqs + (size_t)num_sms;
    uint8_t *b = static_cast<uint8_t *>(ws);
    out->err = reinterpret_cast<uint32_t *>(b);
    b += 256;
    out->counters = reinterpret_cast<uint32_t *>(b);
    b += ((seqs * 4 + 255) / 256) * 256;
    out->slot_ml = reinterpret_cast<float *>(b);
    b += ((slots * n_heads * 2 * 4 + 255) / 256) * 256;
    out->slot_o = reinterpret_cast<float *>(b);
    out->max_slots = slots;
    return true;
}

cudaError_t launch_decode(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group,
                          int grid, cudaStream_t stream) {
    switch (dt) {
        case BML_F32: return launch_d<float>(p, head_dim, group, grid, stream);
        case BML_F16: return launch_d<__half>(p, head_dim, group, grid, stream);
        case BML_BF16: return launch_d<__nv_bfloat16>(p, head_dim, group, grid, stream);
        default: return cudaErrorNotSupported;
    }
}

cudaError_t launch_merge_lse(const float *m, const float *l, const float *o, uint32_t n_parts,
                             uint32_t n_rows, uint32_t head_dim, float *out, cudaStream_t stream) {
    const size_t total = (size_t)n_rows * head_dim;
    if (total == 0) return cudaSuccess;
    const int threads = 256;
    const unsigned blocks = (unsigned)((total + threads - 1) / threads);
    merge_lse_kernel<<<blocks, threads, 0, stream>>>(m, l, o, n_parts, n_rows, head_dim, out);
    return cudaGetLastError();
}

cudaError_t launch_merge_lse_packed(const float *parts, uint32_t n_parts, uint32_t n_rows,
                                    uint32_t head_dim, float *out, cudaStream_t stream) {
    const size_t total = (size_t)n_rows * head_dim;
    if (total == 0) return cudaSuccess;
    const int threads = 256;
    const unsigned blocks = (unsigned)((total + threads - 1) / threads);
    merge_lse_packed_kernel<<<blocks, threads, 0, stream>>>(parts, n_parts, n_rows, head_dim, out);
    return cudaGetLastError();
}

}  // namespace bml
