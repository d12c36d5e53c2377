// decode_tma.cu -- split-K flash decoding for 16-bit KV caches: TMA tile
// loads + warp-level tensor-core MMAs (sm_100a).
//
// Same result, schedule, workspace and merge as decode_mma.cu / decode.cu
// (the attention block of forward_layer_cached,
// crates/compiler/src/gguf_compiler.rs:1008-1050 in SugarFreeDoNoSo/bml, for
// every sequence of a batch) and the same arithmetic as decode_mma.cu
// (m16n8k16 MMAs, q and P as exact pairs of 16-bit terms).  What differs is
// how K and V reach shared memory: per-thread cp.async traffic passes
// through the SM's L1 and tops out near 4.8 TB/s on B200, while the TMA
// engine streams at 6 TB/s.
//
// Each sequence gets two host-encoded tensor maps (K, V) over its cache
// [len][n_kv][D], with the dimensions ordered (d, position, kv head): a box
// of 64 dims x T positions x n_kv heads lands as [head][position][128 B]
// with the 128-byte swizzle keyed on the 128-byte line index, i.e. on the
// position -- so the eight rows of every ldmatrix (eight consecutive
// positions of one head) sit in eight different bank groups, with no
// padding.  (One 4-D box per tile, covering all D dims, measured slightly
// slower than one 3-D box per 64 dims.)  Positions past the
// sequence end are outside the map and arrive as zeros.  Up to 64 sequences
// per launch (the maps travel in the kernel parameters).
//
// Roles: thread 0 fills a 3-stage ring of tiles (T positions, all heads; one
// box per 64 dims of K and of V per tile) on mbarriers; afterwards the last
// warp to finish with a stage refills it (shared-memory counter).  8 warps:
// warp w serves kv head w % n_kv and the 16-position m-tiles w / n_kv
// (mod 8 / n_kv) of every tile, as in decode_mma.cu.
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>
#include <unordered_map>

#include "decode.cuh"
#include "mma_frag.cuh"

namespace bml {

namespace {

constexpr int kSmemBudget = 227 * 1024;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStageK = 32768;  // K bytes of a tile (V the same), as decode.cu
constexpr int kStages = 3;
constexpr int kMaxSeqs = 64;
constexpr float kRescaleThreshold = 8.0f;

struct alignas(64) TmaParams {
    CUtensorMap maps[kMaxSeqs][2];  // K, V of each sequence
    const float *q;
    float *out, *part_m, *part_l, *part_o, *slot_ml, *slot_o;
    uint32_t *counters, *err;
    uint32_t n_seqs, n_heads, n_kv, rows_per_tile, total_tiles, tiles_per_cta, row_bytes;
    float qscale;
    int mode, merge_in_kernel;
    DecodeSeq seqs[kMaxSeqs];
};

template <int D, int G>
struct TCfg {
    static constexpr int NT = (2 * G + 7) / 8;  // n8 column tiles of S (4 heads each)
    static constexpr int KS = D / 16;           // k-steps of S, d-blocks of O^T
    static constexpr int MTW = 128 / D;         // m-tiles per warp per tile
    static constexpr int KB = D / 64;           // boxes (64 dims each) per K or V tile
    static constexpr int STAGE = 2 * kStageK;   // K + V of a tile
    static constexpr int SCR = 64 + 64 + 64;    // barriers [8], counters [8] + cursor, flags
    static constexpr int WSUM = kWarps * G * D * 4;
    static constexpr int WML = kWarps * G * 2 * 4;
    static constexpr int SMEM = kStages * STAGE + SCR + WSUM + WML + 1024;  // + alignment slack
    static_assert(SMEM <= kSmemBudget, "shared memory budget");
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ uint32_t seq_of_tile_t(const TmaParams &p, uint32_t t) {
    uint32_t s = 0;
    while (s + 1 < p.n_seqs && p.seqs[s + 1].tile_begin <= t) ++s;
    return s;
}

__device__ __forceinline__ uint32_t tile_end_of_t(const TmaParams &p, uint32_t s) {
    return s + 1 < p.n_seqs ? p.seqs[s + 1].tile_begin : p.total_tiles;
}

// ----------------------------------------------------------------- kernel
template <int D, int G, bool F16>
__global__ void __launch_bounds__(kThreads, 1) decode_tma_kernel(const __grid_constant__ TmaParams p) {
    using C = TCfg<D, G>;
    constexpr int NT = C::NT, KS = C::KS, MTW = C::MTW, KB = C::KB;
    constexpr float NEG_INF = -INFINITY;

    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t T = p.rows_per_tile;
    const uint32_t box_bytes = p.n_kv * T * 128u;  // one box: n_kv heads x T positions x 128 B
    uint8_t *stages = smem;
    uint8_t *scr = smem + kStages * C::STAGE;
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

    // Ring refill.  Thread 0 fills the ring; afterwards the last warp to
    // finish a stage refills it.  Refills happen in tile order; the cursor
    // (sequence, tile) in cnt[8], cnt[9] is ordered between refillers by
    // every warp's acquire-release increment of every tile's counter.
    auto issue = [&](uint32_t it) {
        uint32_t ps = cnt[8], pt = cnt[9];
        while (pt >= tile_end_of_t(p, ps)) ++ps;
        const uint32_t stage = it % kStages;
        const int row0 = (int)((pt - p.seqs[ps].tile_begin) * T);
        const uint32_t sk = smem_u32(stages + stage * C::STAGE), sv = sk + kStageK;
        uint64_t pol;
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
        mbar_arrive_expect_tx(&full[stage], 2 * KB * box_bytes);
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
            tma_load_3d(sk + kb * box_bytes, &p.maps[ps][0], kb * 64, row0, 0, &full[stage], pol);
            tma_load_3d(sv + kb * box_bytes, &p.maps[ps][1], kb * 64, row0, 0, &full[stage], pol);
        }
        cnt[8] = ps;
        cnt[9] = pt + 1;
    };
    const uint32_t n_tiles = t_end - t_begin;
    if (threadIdx.x == 0) {
        cnt[8] = seq_of_tile_t(p, t_begin);
        cnt[9] = t_begin;
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

    // byte offset of 16-byte chunk `chunk` (0 .. D/8-1) of position `pos`
    // of this warp's head inside a K or V tile: box chunk / 8, 128-byte
    // line (head, pos), 16-byte slot (chunk % 8) ^ (pos % 8)
    const uint32_t head_line = (uint32_t)h * T;
    auto chunk_off = [&](uint32_t pos, uint32_t chunk) {
        const uint32_t line = head_line + pos;
        return (chunk >> 3) * box_bytes + line * 128u + (((chunk & 7u) ^ (pos & 7u)) << 4);
    };

    uint32_t s = seq_of_tile_t(p, t_begin);
    load_q(s);
    bool fresh = true;  // no tile of the current sequence processed yet

    for (uint32_t t = t_begin, it = 0; t < t_end; ++t, ++it) {
        const uint32_t stage = it % kStages;
        mbar_wait(&full[stage], (it / kStages) & 1u, flags, p.err);
        __syncwarp();  // lanes leave the spin separately; ldmatrix and mma need the whole warp
        const uint32_t row0 = (t - p.seqs[s].tile_begin) * T;
        const uint32_t rows = min(T, p.seqs[s].len - row0);
        const uint32_t sk = smem_u32(stages + stage * C::STAGE);
        const uint32_t sv = sk + kStageK;

        // S = K . Qs^T for this warp's m-tiles
        float sc[MTW][NT][4];
#pragma unroll
        for (int mw = 0; mw < MTW; ++mw) {
            const uint32_t mt = (uint32_t)(ph + mw * nph);
            // lane supplies position (lane & 7) + 8 * ((lane >> 3) & 1), chunk lane >> 4
            const uint32_t a_pos = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) sc[mw][nt][i] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t a[4];
                ldsm_x4(sk + chunk_off(a_pos, 2 * ks + (lane >> 4)), a);
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

        // O^T += V^T . P^T  (positions past the end are zero-filled by TMA)
#pragma unroll
        for (int mw = 0; mw < MTW; ++mw) {
            const uint32_t mt = (uint32_t)(ph + mw * nph);
            // lane supplies position (lane & 7) + 8 * (lane >> 4), chunk (lane >> 3) & 1
            const uint32_t v_pos = mt * 16 + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
            for (int db = 0; db < KS; ++db) {
                uint32_t a[4];
                ldsm_x4_t(sv + chunk_off(v_pos, 2 * db + ((lane >> 3) & 1)), a);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816<F16>(o[nt][db], a, pb[mw][nt][0], pb[mw][nt][1]);
            }
        }

        __syncwarp();  // the warp's shared-memory reads of the stage precede lane 0's release
        if (lane == 0) {
            uint32_t old;
            asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                         : "=r"(old)
                         : "r"(smem_u32((const void *)&cnt[stage]))
                         : "memory");
            if (old == (uint32_t)kWarps - 1) {
                cnt[stage] = 0u;
                if (it + kStages < n_tiles) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(it + kStages);
                }
            }
        }

        const bool last_of_cta = (t + 1 == t_end);
        const bool seq_done = (t + 1 == tile_end_of_t(p, s));
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
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// (d, position, kv head) view of one sequence's [len][n_kv][D] 16-bit cache;
// box (64 dims, T positions, n_kv heads), 128-byte swizzle.
bool encode_kv_map(CUtensorMap *map, const void *base, bool f16, uint32_t d, uint32_t n_kv, uint32_t len,
                   uint32_t T) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {d, len, n_kv};
    cuuint64_t strides[2] = {(cuuint64_t)n_kv * d * 2, (cuuint64_t)d * 2};
    cuuint32_t box[3] = {64, T, n_kv};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
               const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, int G, bool F16>
cudaError_t launch_t(const TmaParams &p, int grid, cudaStream_t stream) {
    using C = TCfg<D, G>;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_tma_kernel<D, G, F16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    decode_tma_kernel<D, G, F16><<<grid, kThreads, C::SMEM, stream>>>(p);
    return cudaGetLastError();
}

template <int D, bool F16>
cudaError_t launch_g(const TmaParams &p, uint32_t group, int grid, cudaStream_t stream) {
    switch (group) {
        case 1: return launch_t<D, 1, F16>(p, grid, stream);
        case 2: return launch_t<D, 2, F16>(p, grid, stream);
        case 4: return launch_t<D, 4, F16>(p, grid, stream);
        case 8: return launch_t<D, 8, F16>(p, grid, stream);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace

uint32_t decode_tma_max_seqs() { return kMaxSeqs; }

bool decode_tma_supported(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group) {
    // the warp layout of decode_mma.cu: whole 16-position m-tiles per warp
    return decode_mma_supported(dt, head_dim, n_kv, group) && tensor_map_encoder() != nullptr;
}

cudaError_t launch_decode_tma(const DecodeParams &dp, bml_dtype dt, uint32_t head_dim, uint32_t group, int grid,
                              cudaStream_t stream) {
    if (!decode_tma_supported(dt, head_dim, dp.n_kv, group)) return cudaErrorNotSupported;
    if (dp.n_seqs > (uint32_t)kMaxSeqs || dp.rows_per_tile != kStageK / dp.row_bytes) return cudaErrorInvalidValue;
    static thread_local TmaParams p;  // ~19 KB, kept off the stack
    // Encoding a tensor map is a driver call of a few microseconds; a decode
    // loop that re-submits the same caches (same pointers and lengths) finds
    // its maps here.  Bounded: the cache is dropped when it grows past 4096.
    struct Key {
        const void *k, *v;
        uint32_t len, shape;
        bool operator==(const Key &o) const { return k == o.k && v == o.v && len == o.len && shape == o.shape; }
    };
    struct KeyHash {
        size_t operator()(const Key &x) const {
            return std::hash<const void *>()(x.k) ^ (std::hash<const void *>()(x.v) * 31) ^
                   ((size_t)x.len * 0x9e3779b97f4a7c15ull) ^ x.shape;
        }
    };
    struct Maps {
        CUtensorMap k, v;
    };
    static thread_local std::unordered_map<Key, Maps, KeyHash> cache;
    const bool f16 = dt == BML_F16;
    const uint32_t shape = (head_dim << 16) | (dp.n_kv << 8) | (f16 ? 1u : 0u) | (dp.rows_per_tile << 24);
    for (uint32_t s = 0; s < dp.n_seqs; ++s) {
        const DecodeSeq &e = dp.seqs[s];
        const Key key{e.k, e.v, e.len, shape};
        auto hit = cache.find(key);
        if (hit == cache.end()) {
            Maps m;
            if (!encode_kv_map(&m.k, e.k, f16, head_dim, dp.n_kv, e.len, dp.rows_per_tile) ||
                !encode_kv_map(&m.v, e.v, f16, head_dim, dp.n_kv, e.len, dp.rows_per_tile))
                return cudaErrorNotSupported;
            if (cache.size() >= 4096) cache.clear();
            hit = cache.emplace(key, m).first;
        }
        p.maps[s][0] = hit->second.k;
        p.maps[s][1] = hit->second.v;
        p.seqs[s] = e;
    }
    p.q = dp.q;
    p.out = dp.out;
    p.part_m = dp.part_m;
    p.part_l = dp.part_l;
    p.part_o = dp.part_o;
    p.slot_ml = dp.slot_ml;
    p.slot_o = dp.slot_o;
    p.counters = dp.counters;
    p.err = dp.err;
    p.n_seqs = dp.n_seqs;
    p.n_heads = dp.n_heads;
    p.n_kv = dp.n_kv;
    p.rows_per_tile = dp.rows_per_tile;
    p.total_tiles = dp.total_tiles;
    p.tiles_per_cta = dp.tiles_per_cta;
    p.row_bytes = dp.row_bytes;
    p.qscale = dp.qscale;
    p.mode = dp.mode;
    p.merge_in_kernel = dp.merge_in_kernel;
    if (head_dim == 128) return f16 ? launch_g<128, true>(p, group, grid, stream) : launch_g<128, false>(p, group, grid, stream);
    return f16 ? launch_g<64, true>(p, group, grid, stream) : launch_g<64, false>(p, group, grid, stream);
}

}  // namespace bml
