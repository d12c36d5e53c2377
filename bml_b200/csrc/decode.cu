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
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "decode.cuh"

namespace bml {

namespace {

constexpr int kSmemBudget = 227 * 1024;

// Kernel geometry.  NW warps; warp w serves kv head w % n_kv, the w-th
// "head split" (GW of the G q heads sharing that kv head) and a row phase.
// LPR lanes share one KV row (8 or 16), so a warp step covers RPS = 32/LPR
// rows.
template <typename KT, int D, int G, int GW, int NW, int LPR>
struct Cfg {
    static constexpr int THREADS = NW * 32;
    static constexpr int HS = G / GW;       // head splits per kv head
    static constexpr int RPS = 32 / LPR;    // rows per warp step
    static constexpr int ES = sizeof(KT);
    static constexpr int HEAD_BYTES = D * ES;
    static constexpr int CHUNKS = HEAD_BYTES / 16;
    static constexpr int CPL = CHUNKS / LPR;  // 16-byte chunks per lane
    static constexpr int EPC = 16 / ES;     // elements per chunk
    static constexpr int E = CPL * EPC;     // elements per lane
    static constexpr int E2 = E / 2;        // float2 pairs per lane
    static constexpr int STAGE_K = 32768;   // K bytes per stage; V the same
    // rows per tile T = STAGE_K / (n_kv*HEAD_BYTES); rows per warp = T / nph
    // with nph = NW / (n_kv*HS); RPS rows per warp step.
    static constexpr int STEPS = STAGE_K * HS / (HEAD_BYTES * NW * RPS);
    static constexpr int WSCR = RPS * GW /*alpha*/ + RPS * STEPS * GW /*p*/ + RPS * GW * 2 /*ml*/;
    static constexpr int EXTRA = 2 * 8 * 8 /*barriers*/ + 16 +
                                 4 * (NW * WSCR + NW * GW * D + NW * GW * 2);
    static constexpr int STAGES_FIT = (kSmemBudget - EXTRA) / (2 * STAGE_K);
    static constexpr int STAGES = STAGES_FIT > 4 ? 4 : STAGES_FIT;
    static constexpr int BAR_OFF = STAGES * 2 * STAGE_K;
    static constexpr int SMEM = BAR_OFF + EXTRA;
    static_assert(G % GW == 0, "head split");
    static_assert(LPR == 8 || LPR == 16, "lanes per row");
    static_assert(GW <= LPR, "one owner lane per q head");
    static_assert(CHUNKS % LPR == 0, "head row must be a multiple of LPR 16-byte chunks");
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

// Butterfly reduction of G per-lane partial sums across the LPR lanes of a
// lane group that also transposes: on return, lane j (j = lane % LPR) holds
// the full sum of value index j*G/LPR.
template <int G, int LPR>
__device__ __forceinline__ float transpose_reduce(float (&v)[G], int j) {
    constexpr unsigned FULL = 0xffffffffu;
    constexpr int LEVELS = LPR == 16 ? 4 : 3;
    int n = G;
#pragma unroll
    for (int lvl = 0; lvl < LEVELS; ++lvl) {
        const int mask = (LPR / 2) >> lvl;
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

template <typename KT, int D, int G, int GW, int NW, int LPR>
__global__ void __launch_bounds__(NW * 32, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    using C = Cfg<KT, D, G, GW, NW, LPR>;
    constexpr int STEPS = C::STEPS, E2 = C::E2, CPL = C::CPL, EPC = C::EPC, HS = C::HS, RPS = C::RPS;
    constexpr int HEAD_BYTES = C::HEAD_BYTES, STAGE_K = C::STAGE_K, NST = C::STAGES;
    constexpr int WSCR = C::WSCR, THREADS = C::THREADS;
    constexpr float NEG_INF = -INFINITY;

    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *stages = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    // per stage: warps done with it; [8], [9]: refill cursor (sequence, tile)
    volatile uint32_t *cnt = reinterpret_cast<volatile uint32_t *>(full + 8);
    volatile uint32_t *flags = reinterpret_cast<volatile uint32_t *>(full + 16);
    float *wscr = reinterpret_cast<float *>(smem + C::BAR_OFF + 2 * 8 * 8 + 16);
    float *wsum = wscr + NW * WSCR;  // [NW warps][GW][D]
    float *wml = wsum + NW * GW * D;  // [NW warps][GW][2]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t t_begin = blockIdx.x * p.tiles_per_cta;
    const uint32_t t_end = min(t_begin + p.tiles_per_cta, p.total_tiles);
    const uint32_t T = p.rows_per_tile;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full[i], 1);
            cnt[i] = 0u;
        }
        flags[0] = 0u;
        flags[1] = 0u;
        fence_mbar_init();
    }
    __syncthreads();
    if (t_begin >= t_end) return;

    // Thread 0 fills the ring; afterwards the last warp to finish with a
    // stage refills it (an shared-memory counter per stage), so no warp waits
    // for the others before it starts its next tile.  Refills happen in tile
    // order, so the cursor (sequence, tile) kept in shared memory advances
    // monotonically; each warp's acquire-release increment of every tile's
    // counter orders one refiller's cursor update before the next one's read.
    auto issue = [&](uint32_t it) {
        uint32_t ps = cnt[8], pt = cnt[9];
        while (pt >= tile_end_of(p, ps)) ++ps;
        const uint32_t stage = it % NST;
        const uint32_t row0 = (pt - p.seqs[ps].tile_begin) * T;
        const uint32_t rows = min(T, p.seqs[ps].len - row0);
        const uint32_t bytes = rows * p.row_bytes;
        uint8_t *sk = stages + stage * 2 * STAGE_K;
        const uint64_t pol = l2_policy_evict_first();
        mbar_arrive_expect_tx(&full[stage], 2 * bytes);
        const uint8_t *gk = static_cast<const uint8_t *>(p.seqs[ps].k) + (size_t)row0 * p.row_bytes;
        const uint8_t *gv = static_cast<const uint8_t *>(p.seqs[ps].v) + (size_t)row0 * p.row_bytes;
        bulk_g2s_stream(sk, gk, bytes, &full[stage], pol);
        bulk_g2s_stream(sk + STAGE_K, gv, bytes, &full[stage], pol);
        cnt[8] = ps;
        cnt[9] = pt + 1;
    };
    const uint32_t n_tiles = t_end - t_begin;
    if (threadIdx.x == 0) {
        cnt[8] = seq_of_tile(p, t_begin);
        cnt[9] = t_begin;
        for (uint32_t it = 0; it < n_tiles && it < (uint32_t)NST; ++it) issue(it);
    }

    const int n_kv = (int)p.n_kv;
    const int nph = NW / (n_kv * HS);  // row phases per (kv head, head split)
    const int h = warp % n_kv;
    const int hs = (warp / n_kv) % HS;
    const int ph = warp / (n_kv * HS);
    const int grp = lane / LPR, j = lane % LPR;
    const int own = (j * GW) / LPR;
    const bool owner_lane = (j % (LPR / GW)) == 0;
    float *scr = wscr + warp * WSCR;
    float *s_alpha = scr;                  // [RPS][GW]
    float *s_p = scr + RPS * GW;           // [RPS][STEPS][GW]
    float *s_ml = s_p + RPS * STEPS * GW;  // [RPS][GW][2]

    float2 q2[GW][E2], acc[GW][E2];
    float m_own = NEG_INF, l_own = 0.f;

    uint32_t s = seq_of_tile(p, t_begin);
    auto load_q = [&](uint32_t seq) {
        const float *qs = p.q + ((size_t)seq * p.n_heads + (size_t)h * G + (size_t)hs * GW) * D;
#pragma unroll
        for (int hh = 0; hh < GW; ++hh) {
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                const float4 *src = reinterpret_cast<const float4 *>(qs + hh * D + (j + LPR * c) * EPC);
#pragma unroll
                for (int f = 0; f < EPC / 4; ++f) {
                    const float4 v = __ldg(src + f);
                    q2[hh][(c * EPC) / 2 + 2 * f + 0] = make_float2(v.x * p.qscale, v.y * p.qscale);
                    q2[hh][(c * EPC) / 2 + 2 * f + 1] = make_float2(v.z * p.qscale, v.w * p.qscale);
                }
            }
        }
#pragma unroll
        for (int hh = 0; hh < GW; ++hh)
#pragma unroll
            for (int e = 0; e < E2; ++e) acc[hh][e] = make_float2(0.f, 0.f);
        m_own = NEG_INF;
        l_own = 0.f;
    };
    load_q(s);

    for (uint32_t t = t_begin, it = 0; t < t_end; ++t, ++it) {
        const uint32_t stage = it % NST;
        mbar_wait(&full[stage], (it / NST) & 1u, flags, p.err, p.wait_ns);
        __syncwarp();  // lanes leave the spin separately; the shuffles below need the whole warp
        const uint32_t row0 = (t - p.seqs[s].tile_begin) * T;
        const uint32_t rows = min(T, p.seqs[s].len - row0);
        const uint8_t *sk = stages + stage * 2 * STAGE_K + h * HEAD_BYTES;
        const uint8_t *sv = sk + STAGE_K;

        // pass 1: scores of this lane group's rows (log2 domain)
        float sc[STEPS];
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
            const uint32_t r = (uint32_t)((st * nph + ph) * RPS + grp);
            float2 part2[GW];
#pragma unroll
            for (int hh = 0; hh < GW; ++hh) part2[hh] = make_float2(0.f, 0.f);
            if (r < rows) {
                const uint8_t *rowp = sk + (size_t)r * p.row_bytes;
#pragma unroll
                for (int c = 0; c < CPL; ++c) {
                    const uint4 raw = *reinterpret_cast<const uint4 *>(rowp + (j + LPR * c) * 16);
                    float2 kf[EPC / 2];
                    Elem<KT>::widen2(raw, kf);
#pragma unroll
                    for (int hh = 0; hh < GW; ++hh)
#pragma unroll
                        for (int e = 0; e < EPC / 2; ++e)
                            part2[hh] = __ffma2_rn(q2[hh][c * (EPC / 2) + e], kf[e], part2[hh]);
                }
            }
            float part[GW];
#pragma unroll
            for (int hh = 0; hh < GW; ++hh) part[hh] = part2[hh].x + part2[hh].y;
            const float tot = transpose_reduce<GW, LPR>(part, j);
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
            s_alpha[grp * GW + own] = alpha;
#pragma unroll
            for (int st = 0; st < STEPS; ++st) s_p[(grp * STEPS + st) * GW + own] = sc[st];
        }
        __syncwarp();

        // rescale the accumulators when a running max moved
        float al[GW];
        bool moved = false;
#pragma unroll
        for (int hh = 0; hh < GW; ++hh) {
            al[hh] = s_alpha[grp * GW + hh];
            moved |= (al[hh] != 1.f);
        }
        if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
            for (int hh = 0; hh < GW; ++hh) {
                const float2 a2 = make_float2(al[hh], al[hh]);
#pragma unroll
                for (int e = 0; e < E2; ++e) acc[hh][e] = __fmul2_rn(acc[hh][e], a2);
            }
        }

        // pass 2: P.V
#pragma unroll
        for (int st = 0; st < STEPS; ++st) {
            const uint32_t r = (uint32_t)((st * nph + ph) * RPS + grp);
            if (r < rows) {
                float2 pp[GW];
#pragma unroll
                for (int hh = 0; hh < GW; ++hh) {
                    const float pv = s_p[(grp * STEPS + st) * GW + hh];
                    pp[hh] = make_float2(pv, pv);
                }
                const uint8_t *rowp = sv + (size_t)r * p.row_bytes;
#pragma unroll
                for (int c = 0; c < CPL; ++c) {
                    const uint4 raw = *reinterpret_cast<const uint4 *>(rowp + (j + LPR * c) * 16);
                    float2 vf[EPC / 2];
                    Elem<KT>::widen2(raw, vf);
#pragma unroll
                    for (int hh = 0; hh < GW; ++hh)
#pragma unroll
                        for (int e = 0; e < EPC / 2; ++e)
                            acc[hh][c * (EPC / 2) + e] = __ffma2_rn(pp[hh], vf[e], acc[hh][c * (EPC / 2) + e]);
                }
            }
        }
        __syncwarp();  // the warp's shared-memory reads of the stage precede lane 0's release
        if (lane == 0) {
            uint32_t old;
            asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                         : "=r"(old)
                         : "r"(smem_u32((const void *)&cnt[stage]))
                         : "memory");
            if (old == (uint32_t)NW - 1) {
                cnt[stage] = 0u;
                if (it + NST < n_tiles) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(it + NST);
                }
            }
        }

        const bool last_of_cta = (t + 1 == t_end);
        const bool seq_done = (t + 1 == tile_end_of(p, s));
        if (!(last_of_cta || seq_done)) continue;

        // ---------------------------------------------- finalize sequence s
        if (owner_lane) {
            s_ml[(grp * GW + own) * 2 + 0] = m_own;
            s_ml[(grp * GW + own) * 2 + 1] = l_own;
        }
        __syncwarp();
        float Mh[GW], Lh[GW];
#pragma unroll
        for (int hh = 0; hh < GW; ++hh) {
            float mg[RPS], lg[RPS];
#pragma unroll
            for (int g = 0; g < RPS; ++g) {
                mg[g] = s_ml[(g * GW + hh) * 2 + 0];
                lg[g] = s_ml[(g * GW + hh) * 2 + 1];
            }
            float M = mg[0];
#pragma unroll
            for (int g = 1; g < RPS; ++g) M = fmaxf(M, mg[g]);
            float L = 0.f, mine = 0.f;
#pragma unroll
            for (int g = 0; g < RPS; ++g) {
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
        for (int hh = 0; hh < GW; ++hh)
#pragma unroll
            for (int e = 0; e < E2; ++e) {
#pragma unroll
                for (int m = LPR; m < 32; m <<= 1) {
                    acc[hh][e].x += __shfl_xor_sync(0xffffffffu, acc[hh][e].x, m);
                    acc[hh][e].y += __shfl_xor_sync(0xffffffffu, acc[hh][e].y, m);
                }
            }
        float *ws = wsum + warp * GW * D;
        if (grp == 0) {
#pragma unroll
            for (int hh = 0; hh < GW; ++hh)
#pragma unroll
                for (int c = 0; c < CPL; ++c)
#pragma unroll
                    for (int e = 0; e < EPC / 2; ++e)
                        *reinterpret_cast<float2 *>(ws + hh * D + (j + LPR * c) * EPC + 2 * e) = acc[hh][c * (EPC / 2) + e];
        }
        if (lane == 0) {
#pragma unroll
            for (int hh = 0; hh < GW; ++hh) {
                wml[(warp * GW + hh) * 2 + 0] = Mh[hh];
                wml[(warp * GW + hh) * 2 + 1] = Lh[hh];
            }
        }
        named_bar_sync(1, THREADS);

        const DecodeSeq &sq = p.seqs[s];
        const bool single = (sq.n_slots == 1);
        const uint32_t slot = sq.slot_base + (blockIdx.x - sq.tile_begin / p.tiles_per_cta);
        const uint32_t total = p.n_heads * D;
        const int tid = threadIdx.x;
        for (uint32_t idx = tid; idx < total; idx += THREADS) {
            const uint32_t qh = idx / D, d = idx % D;
            const uint32_t hk = qh / G, hsplit = (qh % G) / GW, hh = qh % GW;
            const int wbase = (int)hk + n_kv * (int)hsplit;  // warp of row phase 0
            float M = NEG_INF;
            for (int w = 0; w < nph; ++w) M = fmaxf(M, wml[((wbase + w * n_kv * HS) * GW + hh) * 2]);
            float L = 0.f, O = 0.f;
            for (int w = 0; w < nph; ++w) {
                const int ww = wbase + w * n_kv * HS;
                const float mw = wml[(ww * GW + hh) * 2];
                const float f = (mw == NEG_INF) ? 0.f : fast_exp2(mw - M);
                L += wml[(ww * GW + hh) * 2 + 1] * f;
                O += wsum[(ww * GW + hh) * D + d] * f;
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
        if (!single && p.merge_in_kernel) {
            __threadfence();
            named_bar_sync(1, THREADS);
            if (tid == 0) {
                const uint32_t old = atomicAdd(&p.counters[s], 1u);
                flags[1] = (old == sq.n_slots - 1) ? 1u : 0u;
            }
            named_bar_sync(1, THREADS);
            if (flags[1]) {
                __threadfence();
                for (uint32_t idx = tid; idx < total; idx += THREADS) {
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
        named_bar_sync(1, THREADS);
        if (!last_of_cta) {
            ++s;
            load_q(s);
        }
    }
}

template <typename KT, int D, int G, int GW, int NW, int LPR>
cudaError_t launch_one(const DecodeParams &p, int grid, cudaStream_t stream) {
    using C = Cfg<KT, D, G, GW, NW, LPR>;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<KT, D, G, GW, NW, LPR>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    decode_kernel<KT, D, G, GW, NW, LPR><<<grid, C::THREADS, C::SMEM, stream>>>(p);
    return cudaGetLastError();
}

// Warp layout per (dtype, head_dim, group).  A KV row is spread over LPR =
// 16 lanes when it has at least 16 chunks of 16 bytes (d=128 16-bit, f32),
// else over 8; each warp carries GW q heads so that q and the accumulators
// fit in the register budget of 16 warps (<= 128 registers a thread).  With
// 16 lanes a row, a group of up to 4 q heads fits in one warp, so every K/V
// element is read from shared memory and widened once.  Shapes whose kv
// heads times head splits exceed 16 warps use 8 warps with all G heads in a
// warp.
template <typename KT, int D, int G>
cudaError_t launch_shape(const DecodeParams &p, int grid, cudaStream_t stream) {
    constexpr int CHUNKS = D * (int)sizeof(KT) / 16;
    constexpr int LPR = CHUNKS >= 16 ? 16 : 8;
    constexpr int E2 = (CHUNKS / LPR) * (16 / (int)sizeof(KT)) / 2;
    constexpr int GW = G <= 1 ? 1 : (G * E2 <= 16 ? G : (16 / E2 >= 1 ? 16 / E2 : 1));
    constexpr int HS = G / GW;
    if ((int)p.n_kv * HS <= 16) return launch_one<KT, D, G, GW, 16, LPR>(p, grid, stream);
    constexpr int E2_8 = (CHUNKS / 8) * (16 / (int)sizeof(KT)) / 2;
    static_assert(E2_8 >= 1, "row too short");
    return launch_one<KT, D, G, G, 8, 8>(p, grid, stream);
}

template <typename KT, int D>
cudaError_t launch_g(const DecodeParams &p, uint32_t group, int grid, cudaStream_t stream) {
    switch (group) {
        case 1: return launch_shape<KT, D, 1>(p, grid, stream);
        case 2: return launch_shape<KT, D, 2>(p, grid, stream);
        case 4: return launch_shape<KT, D, 4>(p, grid, stream);
        case 8: return launch_shape<KT, D, 8>(p, grid, stream);
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

// Merge of a sequence's slots, one CTA per (sequence, head, block of
// 32 * VEC output dims; a row is split into head_dim / (32 * VEC) blocks).
// The slot weights 2^(m_i - M) l_i are computed once per slot in shared
// memory (by every CTA of the row: n_slots x 2 floats); then warp w sums
// slots w, w+8, w+16, ... for the CTA's dims (one 128*VEC-byte load per slot
// and warp, many in flight), and the 8 warp sums are added in warp order --
// a fixed order, so results do not vary between runs.  Few rows (one long
// context) take VEC = 1 for more CTAs; many rows take whole rows per CTA.
template <int VEC>
__global__ void __launch_bounds__(256) slot_merge_kernel(const __grid_constant__ DecodeParams p,
                                                         uint32_t head_dim) {
    __shared__ float w[1024];
    __shared__ float red[8];
    __shared__ float part[8][32 * VEC];
    const uint32_t s = blockIdx.x / p.n_heads, qh = blockIdx.x % p.n_heads;
    const DecodeSeq &sq = p.seqs[s];
    if (sq.n_slots <= 1) return;  // written directly by the decode kernel
    const uint32_t n = min(sq.n_slots, 1024u);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float mx = -INFINITY;
    for (uint32_t i = tid; i < n; i += blockDim.x)
        mx = fmaxf(mx, __ldcg(&p.slot_ml[((size_t)(sq.slot_base + i) * p.n_heads + qh) * 2]));
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float M = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) M = fmaxf(M, red[i]);
    __syncthreads();
    float lsum = 0.f;
    for (uint32_t i = tid; i < n; i += blockDim.x) {
        const size_t sr = (size_t)(sq.slot_base + i) * p.n_heads + qh;
        const float mi = __ldcg(&p.slot_ml[sr * 2]);
        const float f = (mi == -INFINITY) ? 0.f : fast_exp2(mi - M) * __ldcg(&p.slot_ml[sr * 2 + 1]);
        w[i] = f;
        lsum += f;
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, m);
    if (lane == 0) red[warp] = lsum;
    __syncthreads();  // also publishes w[]
    float L = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) L += red[i];
    const uint32_t d0 = (blockIdx.y * 32 + lane) * VEC;
    const size_t stride = (size_t)p.n_heads * head_dim;
    const float *src = p.slot_o + ((size_t)sq.slot_base * p.n_heads + qh) * head_dim + d0;
    float acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = 0.f;
#pragma unroll 8
    for (uint32_t i = warp; i < n; i += 8) {
        const float wi = w[i];
        if constexpr (VEC == 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4 *>(src + i * stride));
            acc[0] += x.x * wi;
            acc[1] += x.y * wi;
            acc[2] += x.z * wi;
            acc[3] += x.w * wi;
        } else if constexpr (VEC == 2) {
            const float2 x = __ldcg(reinterpret_cast<const float2 *>(src + i * stride));
            acc[0] += x.x * wi;
            acc[1] += x.y * wi;
        } else {
            acc[0] += __ldcg(src + i * stride) * wi;
        }
    }
#pragma unroll
    for (int v = 0; v < VEC; ++v) part[warp][lane * VEC + v] = acc[v];
    __syncthreads();
    const size_t row = (size_t)s * p.n_heads + qh;
    for (uint32_t e = tid; e < 32u * VEC; e += blockDim.x) {
        float O = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) O += part[i][e];
        const uint32_t d = blockIdx.y * 32 * VEC + e;
        if (p.mode == kModeFinal) {
            p.out[row * head_dim + d] = O / L;
        } else {
            p.part_o[row * head_dim + d] = O / L;
            if (d == 0) {
                p.part_m[row] = M;
                p.part_l[row] = L;
            }
        }
    }
}

}  // namespace

cudaError_t launch_slot_merge(const DecodeParams &p, uint32_t head_dim, cudaStream_t stream) {
    const unsigned blocks = p.n_seqs * p.n_heads;
    if (blocks == 0) return cudaSuccess;
    if (head_dim % 32 != 0 || head_dim > 128) return cudaErrorInvalidValue;
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (blocks < 2u * (unsigned)sms || head_dim == 32) {
        slot_merge_kernel<1><<<dim3(blocks, head_dim / 32), 256, 0, stream>>>(p, head_dim);
    } else if (head_dim == 64) {
        slot_merge_kernel<2><<<dim3(blocks, 1), 256, 0, stream>>>(p, head_dim);
    } else if (head_dim == 128) {
        slot_merge_kernel<4><<<dim3(blocks, 1), 256, 0, stream>>>(p, head_dim);
    } else {
        slot_merge_kernel<1><<<dim3(blocks, head_dim / 32), 256, 0, stream>>>(p, head_dim);
    }
    return cudaGetLastError();
}

uint32_t decode_rows_per_tile(bml_dtype dt, uint32_t head_dim, uint32_t n_kv) {
    // STAGE_K bytes of K per tile: STEPS * RPS rows for each of the row
    // phases of a kv head
    const uint32_t row_bytes = n_kv * head_dim * (uint32_t)dtype_size(dt);
    return 32768u / row_bytes;
}

// Scratch layout, fixed part first so that calls of any shape agree on it:
//   [0, 64)                   error word (kept until read by a check call)
//   [64, 256)                 claimed-schedule words: CTA exit ticket, merge-
//                             item claims; each call leaves them zero
//   [256, 256 + kTicketBytes) per-sequence counters of a launch (256
//                             sequences at most): tile claims, part
//                             reservations, tiles done (claimed schedule) or
//                             merge tickets (static schedule); each call
//                             leaves them zero
//   [.., + kPartTileBytes)    tiles in each part of the claimed schedule
//                             (kMaxPartTiles words); each call leaves them zero
//   then partial slots of n_heads rows each: as many as the workspace holds,
//   at least 2*seqs + SMs (the static schedule's split points) and one part
//   of every sequence (claimed schedule); the recommended size holds 2*seqs
//   + 8*SMs.
// A shape-dependent counter area would let one call read another call's
// leftover slot values as counters.
constexpr size_t kTicketBytes = (size_t)kMaxSeqsPerLaunch * 8 * 4;
constexpr size_t kPartTileBytes = kMaxPartTiles * 4;

namespace {

constexpr size_t kFixedBytes = 256 + kTicketBytes + kPartTileBytes;

size_t workspace_bytes_for(size_t slots, uint32_t n_heads, uint32_t head_dim) {
    size_t b = kFixedBytes;
    b += ((slots * n_heads * 2 * 4 + 255) / 256) * 256;   // slot (m, l)
    b += slots * n_heads * head_dim * 4;                  // slot o
    return b;
}

size_t launch_seqs(uint32_t n_seqs) { return n_seqs < (uint32_t)kMaxSeqsPerLaunch ? n_seqs : kMaxSeqsPerLaunch; }

}  // namespace

size_t decode_workspace_bytes(uint32_t n_seqs, uint32_t n_heads, uint32_t head_dim, int num_sms) {
    return workspace_bytes_for(std::max<size_t>(2 * launch_seqs(n_seqs) + 8 * (size_t)num_sms,
                                                8 * launch_seqs(n_seqs)),
                               n_heads, head_dim);
}

size_t decode_workspace_min_bytes(uint32_t n_seqs, uint32_t n_heads, uint32_t n_kv, uint32_t head_dim,
                                  int num_sms) {
    // the static schedule's split points, and one part of every sequence of
    // a claimed-schedule launch (one slot per consumer warp of a kv head)
    const size_t nph = n_kv && n_kv <= 8 ? decode_bulk_warps(head_dim) / n_kv : 16;
    return workspace_bytes_for(std::max<size_t>(2 * launch_seqs(n_seqs) + (size_t)num_sms,
                                                nph * launch_seqs(n_seqs)),
                               n_heads, head_dim);
}

size_t decode_workspace_zero_bytes() { return kFixedBytes; }

bool decode_workspace_carve(void *ws, size_t bytes, uint32_t n_seqs, uint32_t n_heads, uint32_t n_kv,
                            uint32_t head_dim, int num_sms, DecodeWorkspace *out) {
    if (!ws || bytes < decode_workspace_min_bytes(n_seqs, n_heads, n_kv, head_dim, num_sms)) return false;
    // the largest slot count whose layout fits in `bytes`
    const size_t per_slot = (size_t)n_heads * (2 + head_dim) * 4;
    size_t slots = (bytes - kFixedBytes - 256) / per_slot;
    while (slots > 0 && workspace_bytes_for(slots, n_heads, head_dim) > bytes) --slots;
    uint8_t *b = static_cast<uint8_t *>(ws);
    out->err = reinterpret_cast<uint32_t *>(b);
    out->sched = reinterpret_cast<uint32_t *>(b + 64);
    b += 256;
    out->counters = reinterpret_cast<uint32_t *>(b);
    b += kTicketBytes;
    out->part_tiles = reinterpret_cast<uint32_t *>(b);
    b += kPartTileBytes;
    out->slot_ml = reinterpret_cast<float *>(b);
    b += ((slots * n_heads * 2 * 4 + 255) / 256) * 256;
    out->slot_o = reinterpret_cast<float *>(b);
    out->max_slots = slots;
    return true;
}

DecodeKernel decode_select(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group) {
    return decode_bulk_supported(dt, head_dim, n_kv, group) ? kKernBulk : kKernCuda;
}

cudaError_t launch_decode(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group, int grid,
                          cudaStream_t stream) {
    switch (dt) {
        case BML_F32: return launch_d<float>(p, head_dim, group, grid, stream);
        case BML_F16: return launch_d<__half>(p, head_dim, group, grid, stream);
        case BML_BF16: return launch_d<__nv_bfloat16>(p, head_dim, group, grid, stream);
        default: return cudaErrorNotSupported;
    }
}

namespace {

// parts [n_parts][n_rows] (m, l) and [n_parts][n_rows][head_dim] o; part i
// weighs c_i 2^(m_i - M) l_i
__global__ void merge_counted_kernel(const float *__restrict__ m, const float *__restrict__ l,
                                     const float *__restrict__ o, uint32_t n_parts, float c0, float c1,
                                     uint32_t n_rows, uint32_t head_dim, float *__restrict__ out) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)n_rows * head_dim) return;
    const uint32_t row = (uint32_t)(idx / head_dim), dd = (uint32_t)(idx % head_dim);
    float M = -INFINITY;
    for (uint32_t i = 0; i < n_parts; ++i) M = fmaxf(M, m[(size_t)i * n_rows + row]);
    float L = 0.f, O = 0.f;
    for (uint32_t i = 0; i < n_parts; ++i) {
        const float mi = m[(size_t)i * n_rows + row];
        const float f = mi == -INFINITY ? 0.f : (i == 0 ? c0 : c1) * fast_exp2(mi - M) * l[(size_t)i * n_rows + row];
        L += f;
        O += o[((size_t)i * n_rows + row) * head_dim + dd] * f;
    }
    out[idx] = O / L;
}

}  // namespace

cudaError_t launch_merge_counted(const float *m, const float *l, const float *o, uint32_t n_parts,
                                 const float *counts, uint32_t n_rows, uint32_t head_dim, float *out,
                                 cudaStream_t stream) {
    if (n_parts == 0 || n_parts > 2) return cudaErrorInvalidValue;
    const size_t total = (size_t)n_rows * head_dim;
    if (total == 0) return cudaSuccess;
    merge_counted_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
        m, l, o, n_parts, counts[0], n_parts > 1 ? counts[1] : 0.f, n_rows, head_dim, out);
    return cudaGetLastError();
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
