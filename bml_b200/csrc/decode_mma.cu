// decode_mma.cu -- split-K flash decoding for 16-bit KV caches with warp-level
// tensor-core MMAs (sm_100a).
//
// Same result as decode.cu (the attention block of forward_layer_cached,
// crates/compiler/src/gguf_compiler.rs:1008-1050 in SugarFreeDoNoSo/bml,
// for every sequence of a batch) and the same schedule, workspace and merge;
// only the arithmetic differs.  Decode reads every K/V byte once and does
// ~4 FLOP per byte, so it is bound by HBM, not by math; what limits a
// CUDA-core kernel is the instruction count per byte (widening, FMAs and
// cross-lane reductions).  Here one m16n8k16 MMA covers 16 positions x 16
// dims of K for all q heads of a group at once, which cuts the instructions
// per KV byte about tenfold.
//
// Precision: q (f32) is written as the sum of two 16-bit terms
// q = q_hi + q_lo + e, |e| <= 2^-16 |q|, which become two columns of the
// MMA's B operand; K is 16-bit already, so S = K.q_hi + K.q_lo carries f32
// products.  P (f32, in [0, 2^8]) is split the same way for P.V.
//
// Tiles and roles:
//  * A tile is T = 32 KiB / row_bytes consecutive positions of one sequence
//    (all kv heads), as in decode.cu.
//  * 8 warps; warp w serves kv head w % n_kv and the 16-position m-tiles
//    m = w / n_kv (mod 8 / n_kv) of every tile.  Each warp streams exactly
//    the bytes it reads -- its head's slice of its m-tiles' rows, K and V --
//    through a private cp.async ring (16-byte copies, L2 evict-first, zero
//    fill past the sequence end), into rows padded by 16 bytes so that the
//    eight row addresses of every ldmatrix fall in different banks.  No warp
//    waits for another between tiles.  Per m-tile:
//      S[16 pos x 8 cols]  = K[16 x D] . Qs^T   (cols = 4 heads x {hi, lo})
//      O^T[D x 8 cols]    += V^T[D x 16] . P^T   (P^T from S's accumulator
//                            registers with one movmatrix transpose)
//    so the softmax of head c lives in the lanes with lane % 4 == c, and
//    each lane's O accumulators belong to its own head: rescaling needs no
//    communication.  A running max moves only when a tile's max exceeds it
//    by more than 2^8 (the final O / l is exact for any fixed reference).
#include <math.h>

#include "decode.cuh"
#include "mma_frag.cuh"

namespace bml {

namespace {

constexpr int kSmemBudget = 227 * 1024;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStageK = 32768;  // K bytes of a tile (V the same), as decode.cu
constexpr float kRescaleThreshold = 8.0f;

template <int D, int G>
struct MCfg {
    static constexpr int NT = (2 * G + 7) / 8;      // n8 column tiles of S (4 heads each)
    static constexpr int KS = D / 16;               // k-steps of S, d-blocks of O^T
    static constexpr int MTW = 128 / D;             // m-tiles per warp per tile
    static constexpr int CPR = D * 2 / 16;          // 16-byte chunks of one head row
    static constexpr int PITCH = D * 2 + 16;        // padded row in a warp's ring
    static constexpr int SLICE = MTW * 16 * PITCH;  // K (or V) rows of one warp, one tile
    static constexpr int WSTAGE = 2 * SLICE;        // K + V
    static constexpr int SCR = 64;                  // flags
    static constexpr int WSUM = kWarps * G * D * 4;  // per-warp partial O [warp][G][D]
    static constexpr int WML = kWarps * G * 2 * 4;   // per-warp (m, l) [warp][G][2]
    static constexpr int EXTRA = SCR + WSUM + WML;
    // Ring depth of a warp: 2.  cp.async data passes through the L1 side of
    // the SM's unified L1 / shared-memory array, so a deeper ring costs
    // streaming rate: measured on B200 (32 x 8192 positions, d=128), 3
    // stages (225 KiB of shared memory) stream at 4.3 TB/s, 2 stages
    // (156 KiB) at 4.8 TB/s.
    static constexpr int NST = 2;
    static constexpr int SMEM = kWarps * NST * WSTAGE + EXTRA;
    static_assert(SMEM <= kSmemBudget, "shared memory budget");
};

// ----------------------------------------------------------------- PTX
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(dst), "l"(src),
                 "r"(src_bytes), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t seq_of_tile_m(const DecodeParams &p, uint32_t t) {
    uint32_t s = 0;
    while (s + 1 < p.n_seqs && p.seqs[s + 1].tile_begin <= t) ++s;
    return s;
}

__device__ __forceinline__ uint32_t tile_end_of_m(const DecodeParams &p, uint32_t s) {
    return s + 1 < p.n_seqs ? p.seqs[s + 1].tile_begin : p.total_tiles;
}

// ----------------------------------------------------------------- kernel
template <int D, int G, bool F16>
__global__ void __launch_bounds__(kThreads, 1) decode_mma_kernel(const __grid_constant__ DecodeParams p) {
    using C = MCfg<D, G>;
    constexpr int NT = C::NT, KS = C::KS, MTW = C::MTW, CPR = C::CPR, PITCH = C::PITCH, NST = C::NST;
    constexpr float NEG_INF = -INFINITY;

    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t row_bytes = p.row_bytes;
    const uint32_t T = p.rows_per_tile;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;  // mma fragment row / column pair
    uint8_t *ring = smem + (size_t)warp * NST * C::WSTAGE;  // this warp's ring
    uint8_t *scr = smem + (size_t)kWarps * NST * C::WSTAGE;
    volatile uint32_t *flags = reinterpret_cast<volatile uint32_t *>(scr);
    float *wsum = reinterpret_cast<float *>(scr + C::SCR);  // [warp][G][D]
    float *wml = wsum + kWarps * G * D;                     // [warp][G][2]
    const uint32_t t_begin = blockIdx.x * p.tiles_per_cta;
    const uint32_t t_end = min(t_begin + p.tiles_per_cta, p.total_tiles);
    if (threadIdx.x == 0) {
        flags[0] = 0u;
        flags[1] = 0u;
    }
    __syncthreads();
    if (t_begin >= t_end) return;

    const int n_kv = (int)p.n_kv;
    const int nph = kWarps / n_kv;  // warps per kv head
    const int h = warp % n_kv, ph = warp / n_kv;
    const uint64_t pol = l2_policy_evict_first();
    const uint32_t ring_a = smem_u32(ring);

    // Copies this warp's rows of tile t (sequence ps) into ring stage st:
    // lane l moves chunk l % CPR of rows l / CPR + k * (32 / CPR); rows past
    // the sequence end are zero-filled.
    auto fetch = [&](uint32_t t, uint32_t ps, uint32_t st) {
        const DecodeSeq &q = p.seqs[ps];
        const uint32_t row0 = (t - q.tile_begin) * T;
        const uint32_t chunk = (uint32_t)lane % CPR;
        const uint8_t *kb = static_cast<const uint8_t *>(q.k) + (size_t)h * D * 2 + chunk * 16;
        const uint8_t *vb = static_cast<const uint8_t *>(q.v) + (size_t)h * D * 2 + chunk * 16;
        const uint32_t dk = ring_a + st * C::WSTAGE + chunk * 16, dv = dk + C::SLICE;
#pragma unroll
        for (int k = 0; k < MTW * 16 * CPR / 32; ++k) {
            const uint32_t wr = (uint32_t)lane / CPR + k * (32 / CPR);  // row within the warp's slice
            const uint32_t pos = row0 + (uint32_t)(ph + (wr / 16) * nph) * 16 + wr % 16;
            const bool ok = pos < q.len;
            const size_t off = ok ? (size_t)pos * row_bytes : 0;
            cp_async16(dk + wr * PITCH, kb + off, ok ? 16u : 0u, pol);
            cp_async16(dv + wr * PITCH, vb + off, ok ? 16u : 0u, pol);
        }
    };

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

    uint32_t s = seq_of_tile_m(p, t_begin);
    load_q(s);
    bool fresh = true;  // no tile of the current sequence processed yet

    // prologue: tiles t_begin .. t_begin + NST - 2 in flight
    uint32_t fs = s, ft = t_begin;  // fetch cursor
    auto fetch_next = [&](uint32_t st) {
        if (ft < t_end) {
            while (ft >= tile_end_of_m(p, fs)) ++fs;
            fetch(ft, fs, st);
            ++ft;
        }
        cp_async_commit();  // one group per ring slot, empty past the end
    };
#pragma unroll
    for (int i = 0; i < NST - 1; ++i) fetch_next((uint32_t)i);

    for (uint32_t t = t_begin, it = 0; t < t_end; ++t, ++it) {
        const uint32_t stage = it % NST;
        // refill the slot of tile it - 1 (read by this warp last iteration)
        fetch_next((it + NST - 1) % NST);
        cp_async_wait<NST - 1>();  // this lane's copies of tile it have landed
        __syncwarp();              // ... and every lane's
        const uint32_t row0 = (t - p.seqs[s].tile_begin) * T;
        const uint32_t rows = min(T, p.seqs[s].len - row0);
        const uint32_t sk = ring_a + stage * C::WSTAGE;
        const uint32_t sv = sk + C::SLICE;

        // S = K . Qs^T for this warp's m-tiles
        float sc[MTW][NT][4];
#pragma unroll
        for (int mw = 0; mw < MTW; ++mw) {
            // lane supplies row (lane & 7) + 8 * ((lane >> 3) & 1), chunk lane >> 4
            const uint32_t a_row = (uint32_t)mw * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            const uint32_t a_base = sk + a_row * PITCH + (lane >> 4) * 16;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) sc[mw][nt][i] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t a[4];
                ldsm_x4(a_base + ks * 32, a);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816<F16>(sc[mw][nt], a, qb[nt][ks][0], qb[nt][ks][1]);
            }
        }

        // softmax: lane (g, c) holds head nt*4 + c at positions g and g + 8
        // of each m-tile; the heads' tile maxima need lanes xor 4, 8, 16
        float sv_[MTW][NT][2];
        float alpha[NT], m_use[NT];
        bool moved = false;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float mx = NEG_INF;
#pragma unroll
            for (int mw = 0; mw < MTW; ++mw) {
                const uint32_t r = (uint32_t)(ph + mw * nph) * 16 + g;
                sv_[mw][nt][0] = r < rows ? sc[mw][nt][0] + sc[mw][nt][1] : NEG_INF;
                sv_[mw][nt][1] = r + 8 < rows ? sc[mw][nt][2] + sc[mw][nt][3] : NEG_INF;
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

        // O^T += V^T . P^T
        const bool partial = rows < T;
#pragma unroll
        for (int mw = 0; mw < MTW; ++mw) {
            const uint32_t mt = (uint32_t)(ph + mw * nph);
            // lane supplies row (lane & 7) + 8 * (lane >> 4), chunk (lane >> 3) & 1
            const uint32_t v_row = (uint32_t)mw * 16 + (lane & 7) + (lane >> 4) * 8;
            const uint32_t v_base = sv + v_row * PITCH + ((lane >> 3) & 1) * 16;
            // positions of this lane's A elements: 2c, 2c+1 (a0, a1), +8 (a2, a3)
            const uint32_t p0 = mt * 16 + 2 * c;
            const uint32_t keep_lo = partial ? ((p0 < rows ? 0x0000ffffu : 0u) | (p0 + 1 < rows ? 0xffff0000u : 0u))
                                             : 0xffffffffu;
            const uint32_t keep_hi = partial ? ((p0 + 8 < rows ? 0x0000ffffu : 0u) |
                                                (p0 + 9 < rows ? 0xffff0000u : 0u))
                                             : 0xffffffffu;
#pragma unroll
            for (int db = 0; db < KS; ++db) {
                uint32_t a[4];
                ldsm_x4_t(v_base + db * 32, a);
                a[0] &= keep_lo;
                a[1] &= keep_lo;
                a[2] &= keep_hi;
                a[3] &= keep_hi;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816<F16>(o[nt][db], a, pb[mw][nt][0], pb[mw][nt][1]);
            }
        }

        __syncwarp();  // every lane's reads of this slot precede its refill next iteration

        const bool last_of_cta = (t + 1 == t_end);
        const bool seq_done = (t + 1 == tile_end_of_m(p, s));
        if (!(last_of_cta || seq_done)) continue;

        // ---------------------------------------------- finalize sequence s
        // per head: l over the 8 lanes of the head, then this warp's partial
        // (unnormalised O relative to m, m, l) into shared memory
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

template <int D, int G, bool F16>
cudaError_t launch_t(const DecodeParams &p, int grid, cudaStream_t stream) {
    using C = MCfg<D, G>;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_mma_kernel<D, G, F16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    decode_mma_kernel<D, G, F16><<<grid, kThreads, C::SMEM, stream>>>(p);
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

}  // namespace

bool decode_mma_supported(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group) {
    if (dt != BML_BF16 && dt != BML_F16) return false;
    if (head_dim != 64 && head_dim != 128) return false;
    if (group != 1 && group != 2 && group != 4 && group != 8) return false;
    if (n_kv != 1 && n_kv != 2 && n_kv != 4 && n_kv != 8) return false;
    // whole m-tiles: T = 32 KiB / row_bytes must be a multiple of 16 and
    // split evenly over the 8 / n_kv warps of a kv head
    const uint32_t row_bytes = n_kv * head_dim * 2;
    if (row_bytes < 512 || row_bytes > 2048) return false;
    const uint32_t T = kStageK / row_bytes;
    return T % 16 == 0 && (T / 16) % (kWarps / n_kv) == 0;
}

cudaError_t launch_decode_mma(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group, int grid,
                              cudaStream_t stream) {
    if (!decode_mma_supported(dt, head_dim, p.n_kv, group)) return cudaErrorNotSupported;
    if (p.rows_per_tile != kStageK / p.row_bytes) return cudaErrorInvalidValue;
    const bool f16 = dt == BML_F16;
    if (head_dim == 128) return f16 ? launch_g<128, true>(p, group, grid, stream) : launch_g<128, false>(p, group, grid, stream);
    return f16 ? launch_g<64, true>(p, group, grid, stream) : launch_g<64, false>(p, group, grid, stream);
}

}  // namespace bml
