// decode_bulk.cu -- split-K flash decoding for 16-bit KV caches: 1-D bulk
// copies of whole cache rows + warp-level tensor-core MMAs (sm_100a).
//
// Same result, schedule, workspace and merge as decode.cu / decode_mma.cu /
// decode_tma.cu (the attention block of forward_layer_cached,
// crates/compiler/src/gguf_compiler.rs:1008-1050 in SugarFreeDoNoSo/bml, for
// every sequence of a batch) and the same arithmetic as decode_mma.cu
// (m16n8k16 MMAs, q and P as exact pairs of 16-bit terms).  What differs is
// how K and V reach shared memory.
//
// A tile of T positions of a cache ([len][n_kv][D], row_bytes = n_kv*D*2
// contiguous bytes per position) arrives as eight 1-D bulk copies, one per
// group of Gc = T/8 consecutive positions, each group landing 16 bytes
// further along modulo 128 than the one before (group pitch Gc*row_bytes +
// 16).  The MMA row order inside a 16-position m-tile is free (the softmax
// and P.V only need to agree on it), so m-tile mt's row r is position
// (r % 8) * Gc + 2*mt + r / 8: the eight rows of every ldmatrix come from
// eight different groups and hit eight different bank groups.  Large plain
// bulk copies stream faster than tensor-map tile loads with 128-byte boxes,
// need no host-encoded tensor map (no per-length encode, 256 sequences a
// launch like the other kernels), and read nothing past a sequence's last
// position: the rows of a partial last tile that are not copied keep stale
// bytes, whose scores are masked and whose V elements are zeroed in the MMA
// fragments.
//
// Roles: warp 0 fills a 3-stage ring of tiles (T positions, all heads); the
// last warp to finish with a stage refills it, lanes 0-7 issuing the K group
// copies and lanes 8-15 the V ones.  8 warps: warp w serves kv head w % n_kv and the
// 16-position m-tiles w / n_kv (mod 8 / n_kv) of every tile, as in
// decode_mma.cu.
#include <math.h>

#include "decode.cuh"
#include "mma_frag.cuh"

namespace bml {

namespace {

constexpr int kSmemBudget = 227 * 1024;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStageK = 32768;  // K bytes of a full tile (V the same), as decode.cu
constexpr int kStages = 3;
constexpr float kRescaleThreshold = 8.0f;

template <int D, int G>
struct BCfg {
    static constexpr int NT = (2 * G + 7) / 8;  // n8 column tiles of S (4 heads each)
    static constexpr int KS = D / 16;           // k-steps of S, d-blocks of O^T
    static constexpr int MTW = 128 / D;         // m-tiles per warp per tile
    static constexpr int SCR = 64 + 64 + 64;    // barriers [8], counters [8] + cursor, flags
    static constexpr int WSUM = kWarps * G * D * 4;
    static constexpr int WML = kWarps * G * 2 * 4;
};

// Bytes of one K (or V) tile of T rows: eight groups at pitch
// (T/8)*row_bytes + 16 (row_bytes is a multiple of 128).
__host__ __device__ __forceinline__ uint32_t ktile_bytes_of(uint32_t T, uint32_t row_bytes) {
    return T * row_bytes + 128u;
}

template <int D, int G>
uint32_t smem_bytes(uint32_t T, uint32_t row_bytes) {
    using C = BCfg<D, G>;
    return kStages * 2u * ktile_bytes_of(T, row_bytes) + C::SCR + C::WSUM + C::WML + 128u;
}

__device__ __forceinline__ uint32_t seq_of_tile_b(const DecodeParams &p, uint32_t t) {
    uint32_t s = 0;
    while (s + 1 < p.n_seqs && p.seqs[s + 1].tile_begin <= t) ++s;
    return s;
}

__device__ __forceinline__ uint32_t tile_end_of_b(const DecodeParams &p, uint32_t s) {
    return s + 1 < p.n_seqs ? p.seqs[s + 1].tile_begin : p.total_tiles;
}

// ----------------------------------------------------------------- kernel
template <int D, int G, bool F16>
__global__ void __launch_bounds__(kThreads, 1) decode_bulk_kernel(const __grid_constant__ DecodeParams p) {
    using C = BCfg<D, G>;
    constexpr int NT = C::NT, KS = C::KS, MTW = C::MTW;
    constexpr float NEG_INF = -INFINITY;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_addr + 127u) & ~127u) - raw_addr);
    const uint32_t T = p.rows_per_tile;
    const uint32_t row_bytes = p.row_bytes;
    const uint32_t gc = T / 8u;                       // positions per copy group
    const uint32_t gpitch = gc * row_bytes + 16u;     // group pitch in shared memory
    const uint32_t ktile_bytes = ktile_bytes_of(T, row_bytes);
    const uint32_t stage_bytes = 2u * ktile_bytes;
    uint8_t *stages = smem;
    uint8_t *scr = smem + kStages * stage_bytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(scr);                        // [8]
    volatile uint32_t *cnt = reinterpret_cast<volatile uint32_t *>(full + 8);  // [8], cursor [8], [9]
    volatile uint32_t *flags = reinterpret_cast<volatile uint32_t *>(full + 16);
    float *wsum = reinterpret_cast<float *>(scr + C::SCR);  // [warp][G][D]
    float *wml = wsum + kWarps * G * D;                     // [warp][G][2]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;  // mma fragment row / column pair
    const uint32_t t_begin = blockIdx.x * p.tiles_per_cta;
    const uint32_t t_end = min(t_begin + p.tiles_per_cta, p.total_tiles);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            cnt[i] = 0u;
        }
        flags[0] = 0u;
        flags[1] = 0u;
        fence_mbar_init();
    }
    __syncthreads();
    if (t_begin >= t_end) return;

    // Ring refill by one whole (converged) warp.  Warp 0 fills the ring;
    // afterwards the last warp to finish a stage refills it.  Refills happen
    // in tile order; lane 0 keeps the cursor (sequence, tile) in cnt[8],
    // cnt[9], ordered between refillers by every warp's acquire-release
    // increment (lane 0) of every tile's counter.
    auto issue = [&](uint32_t it) {
        uint32_t ps = 0, pt = 0;
        if (lane == 0) {
            ps = cnt[8];
            pt = cnt[9];
            while (pt >= tile_end_of_b(p, ps)) ++ps;
        }
        ps = __shfl_sync(0xffffffffu, ps, 0);
        pt = __shfl_sync(0xffffffffu, pt, 0);
        __syncwarp();
        const uint32_t stage = it % kStages;
        const DecodeSeq &sq = p.seqs[ps];
        const uint32_t row0 = (pt - sq.tile_begin) * T;
        const uint32_t rows = min(T, sq.len - row0);
        uint8_t *sk = stages + stage * stage_bytes;
        if (lane == 0) mbar_arrive_expect_tx(&full[stage], 2u * rows * row_bytes);
        __syncwarp();  // expected bytes are posted before any copy can complete
        // the generic-proxy reads of this stage (every warp's ldmatrix,
        // ordered here by the counter) precede the async-proxy writes
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const uint64_t pol = l2_policy_evict_first();
        const uint8_t *gk = static_cast<const uint8_t *>(sq.k) + (size_t)row0 * row_bytes;
        const uint8_t *gv = static_cast<const uint8_t *>(sq.v) + (size_t)row0 * row_bytes;
        if (lane < 16) {
            const uint32_t j = lane & 7u;  // group
            const uint32_t n = rows > j * gc ? min(gc, rows - j * gc) : 0u;
            if (n) {
                const uint8_t *src = (lane < 8 ? gk : gv) + (size_t)j * gc * row_bytes;
                bulk_g2s_stream(sk + (lane < 8 ? 0u : ktile_bytes) + j * gpitch, src, n * row_bytes, &full[stage],
                                pol);
            }
        }
        if (lane == 0) {
            cnt[8] = ps;
            cnt[9] = pt + 1;
        }
        __syncwarp();
    };
    const uint32_t n_tiles = t_end - t_begin;
    if (warp == 0) {
        if (lane == 0) {
            cnt[8] = seq_of_tile_b(p, t_begin);
            cnt[9] = t_begin;
        }
        __syncwarp();
        for (uint32_t it = 0; it < n_tiles && it < (uint32_t)kStages; ++it) issue(it);
    }

    const int n_kv = (int)p.n_kv;
    const int nph = kWarps / n_kv;  // warps per kv head
    const int h = warp % n_kv, ph = warp / n_kv;

    // q of the group as the MMA's B operand: column n = 2*head + term.
    uint32_t qb[NT][KS][2];
    float o[NT][KS][4];
    float m_run[NT], l_part[NT];
    auto load_q = [&](uint32_t seq) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int n = nt * 8 + g;
            const int hd = n >> 1, term = n & 1;
            const float *qs = p.q + ((size_t)seq * p.n_heads + (size_t)h * G + (hd < G ? hd : 0)) * D;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t w = 0;
                    if (hd < G) {
                        const float2 v = *reinterpret_cast<const float2 *>(qs + ks * 16 + half * 8 + 2 * c);
                        w = (uint32_t)term16<F16>(v.x * p.qscale, term) |
                            ((uint32_t)term16<F16>(v.y * p.qscale, term) << 16);
                    }
                    qb[nt][ks][half] = w;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) o[nt][ks][i] = 0.f;
            }
            m_run[nt] = NEG_INF;
            l_part[nt] = 0.f;
        }
    };

    // byte offset of 16-byte chunk `chunk` (0 .. D/8-1) of this warp's head
    // at row r (0..15) of m-tile mt, i.e. position (r % 8) * gc + 2*mt + r / 8
    const uint32_t head_off = (uint32_t)h * D * 2u;
    auto chunk_off = [&](uint32_t mt, uint32_t r, uint32_t chunk) {
        return (r & 7u) * gpitch + (2u * mt + (r >> 3)) * row_bytes + head_off + (chunk << 4);
    };
    auto pos_of = [&](uint32_t mt, uint32_t r) { return (r & 7u) * gc + 2u * mt + (r >> 3); };

    uint32_t s = seq_of_tile_b(p, t_begin);
    load_q(s);
    bool fresh = true;  // no tile of the current sequence processed yet

    for (uint32_t t = t_begin, it = 0; t < t_end; ++t, ++it) {
        const uint32_t stage = it % kStages;
        mbar_wait(&full[stage], (it / kStages) & 1u, flags, p.err);
        __syncwarp();  // lanes leave the spin separately; ldmatrix and mma need the whole warp
        const uint32_t row0 = (t - p.seqs[s].tile_begin) * T;
        const uint32_t rows = min(T, p.seqs[s].len - row0);
        const uint32_t sk = smem_u32(stages + stage * stage_bytes);
        const uint32_t sv = sk + ktile_bytes;
        const bool partial = rows < T;  // rows past the end hold stale bytes

        // S = K . Qs^T for this warp's m-tiles
        float sc[MTW][NT][4];
#pragma unroll
        for (int mw = 0; mw < MTW; ++mw) {
            const uint32_t mt = (uint32_t)(ph + mw * nph);
            // lane supplies row (lane & 7) + 8 * ((lane >> 3) & 1), chunk lane >> 4
            const uint32_t a_row = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) sc[mw][nt][i] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t a[4];
                ldsm_x4(sk + chunk_off(mt, a_row, 2 * ks + (lane >> 4)), a);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816<F16>(sc[mw][nt], a, qb[nt][ks][0], qb[nt][ks][1]);
            }
        }

        // softmax: lane (g, c) holds head nt*4 + c at rows g and g + 8 of
        // each m-tile; the heads' tile maxima need lanes xor 4, 8, 16
        float sv_[MTW][NT][2];
        float alpha[NT], m_use[NT];
        bool moved = false;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float mx = NEG_INF;
#pragma unroll
            for (int mw = 0; mw < MTW; ++mw) {
                const uint32_t mt = (uint32_t)(ph + mw * nph);
                sv_[mw][nt][0] = pos_of(mt, g) < rows ? sc[mw][nt][0] + sc[mw][nt][1] : NEG_INF;
                sv_[mw][nt][1] = pos_of(mt, g + 8) < rows ? sc[mw][nt][2] + sc[mw][nt][3] : NEG_INF;
                mx = fmax3(mx, sv_[mw][nt][0], sv_[mw][nt][1]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            float mn = m_run[nt];
            if (m_run[nt] == NEG_INF || mx > m_run[nt] + kRescaleThreshold) mn = fmaxf(m_run[nt], mx);
            m_use[nt] = mn == NEG_INF ? 0.f : mn;
            alpha[nt] = m_run[nt] == NEG_INF ? 0.f : fast_exp2(m_run[nt] - m_use[nt]);
            moved |= !fresh && mn != m_run[nt];
            m_run[nt] = mn;
        }
        if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                    for (int i = 0; i < 4; ++i) o[nt][ks][i] *= alpha[nt];
        }
        fresh = false;

        // P -> (hi, lo) 16-bit pairs, transposed into the B operand of P.V
        uint32_t pb[MTW][NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float lsum = 0.f;
#pragma unroll
            for (int mw = 0; mw < MTW; ++mw) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const float x = sv_[mw][nt][half];
                    const float pv = x == NEG_INF ? 0.f : fast_exp2(x - m_use[nt]);
                    lsum += pv;
                    pb[mw][nt][half] = movm_t(split2<F16>(pv));
                }
            }
            l_part[nt] = l_part[nt] * alpha[nt] + lsum;
        }

        // O^T += V^T . P^T.  Rows past the sequence end were not copied: P
        // is 0 there, and their V elements are zeroed in the fragments (the
        // stale bytes may hold any bit pattern, NaN included).
#pragma unroll
        for (int mw = 0; mw < MTW; ++mw) {
            const uint32_t mt = (uint32_t)(ph + mw * nph);
            // lane supplies row (lane & 7) + 8 * (lane >> 4), chunk (lane >> 3) & 1
            const uint32_t v_row = (lane & 7) + (lane >> 4) * 8;
            // after the transpose, a[0], a[1] hold rows 2c, 2c+1 and a[2],
            // a[3] rows 2c+8, 2c+9 (low, high half)
            uint32_t keep01 = 0xffffffffu, keep23 = 0xffffffffu;
            if (partial) {
                const uint32_t r0 = 2 * c;
                keep01 = (pos_of(mt, r0) < rows ? 0x0000ffffu : 0u) | (pos_of(mt, r0 + 1) < rows ? 0xffff0000u : 0u);
                keep23 = (pos_of(mt, r0 + 8) < rows ? 0x0000ffffu : 0u) |
                         (pos_of(mt, r0 + 9) < rows ? 0xffff0000u : 0u);
            }
#pragma unroll
            for (int db = 0; db < KS; ++db) {
                uint32_t a[4];
                ldsm_x4_t(sv + chunk_off(mt, v_row, 2 * db + ((lane >> 3) & 1)), a);
                a[0] &= keep01;
                a[1] &= keep01;
                a[2] &= keep23;
                a[3] &= keep23;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816<F16>(o[nt][db], a, pb[mw][nt][0], pb[mw][nt][1]);
            }
        }

        __syncwarp();  // the warp's shared-memory reads of the stage precede lane 0's release
        uint32_t old = 0;
        if (lane == 0)
            asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                         : "=r"(old)
                         : "r"(smem_u32((const void *)&cnt[stage]))
                         : "memory");
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == (uint32_t)kWarps - 1) {  // warp-uniform: this warp refills the stage
            if (lane == 0) cnt[stage] = 0u;
            if (it + kStages < n_tiles) issue(it + kStages);
        }

        const bool last_of_cta = (t + 1 == t_end);
        const bool seq_done = (t + 1 == tile_end_of_b(p, s));
        if (!(last_of_cta || seq_done)) continue;

        // ---------------------------------------------- finalize sequence s
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float L = l_part[nt];
            L += __shfl_xor_sync(0xffffffffu, L, 4);
            L += __shfl_xor_sync(0xffffffffu, L, 8);
            L += __shfl_xor_sync(0xffffffffu, L, 16);
            const int hd = nt * 4 + c;
            if (hd < G) {
                float *ws = wsum + ((size_t)warp * G + hd) * D;
#pragma unroll
                for (int db = 0; db < KS; ++db) {
                    ws[db * 16 + g] = o[nt][db][0] + o[nt][db][1];
                    ws[db * 16 + g + 8] = o[nt][db][2] + o[nt][db][3];
                }
                if (g == 0) {
                    wml[(warp * G + hd) * 2 + 0] = m_run[nt];
                    wml[(warp * G + hd) * 2 + 1] = L;
                }
            }
        }
        named_bar_sync(1, kThreads);

        const DecodeSeq &sq = p.seqs[s];
        const bool single = (sq.n_slots == 1);
        const uint32_t slot = sq.slot_base + (blockIdx.x - sq.tile_begin / p.tiles_per_cta);
        const uint32_t total = p.n_heads * D;
        const int tid = threadIdx.x;
        for (uint32_t idx = tid; idx < total; idx += kThreads) {
            const uint32_t qh = idx / D, d = idx % D;
            const uint32_t hk = qh / G, hh = qh % G;
            float M = NEG_INF;
            for (int w = 0; w < nph; ++w) M = fmaxf(M, wml[(((int)hk + w * n_kv) * G + hh) * 2]);
            float L = 0.f, O = 0.f;
            for (int w = 0; w < nph; ++w) {
                const int ww = (int)hk + w * n_kv;
                const float mw = wml[(ww * G + hh) * 2];
                const float f = (mw == NEG_INF) ? 0.f : fast_exp2(mw - M);
                L += wml[(ww * G + hh) * 2 + 1] * f;
                O += wsum[(ww * G + hh) * D + d] * f;
            }
            const float ov = O / L;
            const size_t row = (size_t)s * p.n_heads + qh;
            if (single) {
                if (p.mode == kModeFinal) {
                    p.out[row * D + d] = ov;
                } else {
                    p.part_o[row * D + d] = ov;
                    if (d == 0) {
                        p.part_m[row] = M;
                        p.part_l[row] = L;
                    }
                }
            } else {
                p.slot_o[((size_t)slot * p.n_heads + qh) * D + d] = ov;
                if (d == 0) {
                    p.slot_ml[((size_t)slot * p.n_heads + qh) * 2 + 0] = M;
                    p.slot_ml[((size_t)slot * p.n_heads + qh) * 2 + 1] = L;
                }
            }
        }
        if (!single && p.merge_in_kernel) {
            __threadfence();
            named_bar_sync(1, kThreads);
            if (tid == 0) {
                const uint32_t old = atomicAdd(&p.counters[s], 1u);
                flags[1] = (old == sq.n_slots - 1) ? 1u : 0u;
            }
            named_bar_sync(1, kThreads);
            if (flags[1]) {
                __threadfence();
                for (uint32_t idx = tid; idx < total; idx += kThreads) {
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
        named_bar_sync(1, kThreads);
        if (!last_of_cta) {
            ++s;
            load_q(s);
            fresh = true;
        }
    }
}

// ----------------------------------------------------------------- host
template <int D, int G, bool F16>
cudaError_t launch_t(const DecodeParams &p, int grid, cudaStream_t stream) {
    const uint32_t smem = smem_bytes<D, G>(p.rows_per_tile, p.row_bytes);
    if (smem > (uint32_t)kSmemBudget) return cudaErrorNotSupported;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_bulk_kernel<D, G, F16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    decode_bulk_kernel<D, G, F16><<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

template <int D, bool F16>
cudaError_t launch_g(const DecodeParams &p, uint32_t group, int grid, cudaStream_t stream) {
    switch (group) {
        case 1: return launch_t<D, 1, F16>(p, grid, stream);
        case 2: return launch_t<D, 2, F16>(p, grid, stream);
        case 4: return launch_t<D, 4, F16>(p, grid, stream);
        case 8: return launch_t<D, 8, F16>(p, grid, stream);
        default: return cudaErrorNotSupported;
    }
}

template <int D>
uint32_t smem_for_group(uint32_t group, uint32_t T, uint32_t row_bytes) {
    switch (group) {
        case 1: return smem_bytes<D, 1>(T, row_bytes);
        case 2: return smem_bytes<D, 2>(T, row_bytes);
        case 4: return smem_bytes<D, 4>(T, row_bytes);
        default: return smem_bytes<D, 8>(T, row_bytes);
    }
}

}  // namespace

bool decode_bulk_supported(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group) {
    // the warp layout of decode_mma.cu, and the padded ring within 227 KB
    if (!decode_mma_supported(dt, head_dim, n_kv, group)) return false;
    const uint32_t T = decode_rows_per_tile(dt, head_dim, n_kv);
    const uint32_t row_bytes = n_kv * head_dim * 2u;
    const uint32_t smem = head_dim == 128 ? smem_for_group<128>(group, T, row_bytes)
                                          : smem_for_group<64>(group, T, row_bytes);
    return smem <= (uint32_t)kSmemBudget;
}

cudaError_t launch_decode_bulk(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group, int grid,
                               cudaStream_t stream) {
    if (!decode_bulk_supported(dt, head_dim, p.n_kv, group)) return cudaErrorNotSupported;
    if (p.rows_per_tile * p.row_bytes > (uint32_t)kStageK || p.row_bytes % 16 != 0) return cudaErrorInvalidValue;
    const bool f16 = dt == BML_F16;
    if (head_dim == 128) return f16 ? launch_g<128, true>(p, group, grid, stream) : launch_g<128, false>(p, group, grid, stream);
    return f16 ? launch_g<64, true>(p, group, grid, stream) : launch_g<64, false>(p, group, grid, stream);
}

}  // namespace bml
