// decode_bulk.cu -- split-K flash decoding for 16-bit KV caches: group bulk
// copies + warp-level tensor-core MMAs, with chunks of work claimed at run
// time (sm_100a).
//
// Same result and arithmetic as decode_mma.cu / decode_tma.cu (the attention
// block of forward_layer_cached, crates/compiler/src/gguf_compiler.rs:
// 1008-1050 in SugarFreeDoNoSo/bml, for every sequence of a batch; m16n8k16
// MMAs with q and P as exact pairs of 16-bit terms).  What differs is how K
// and V reach shared memory and how the work is spread over the SMs.
//
// Loads.  A tile of T positions of a cache ([len][n_kv][D], row_bytes =
// n_kv*D*2 contiguous bytes per position) arrives as eight 1-D bulk copies,
// one per group of Gc = T/8 consecutive positions, each group landing 16
// bytes further along modulo 128 than the one before (group pitch
// Gc*row_bytes + 16).  The MMA row order inside a 16-position m-tile is free
// (the softmax and P.V only need to agree on it), so m-tile mt's row r is
// position (r % 8) * Gc + 2*mt + r / 8: the eight rows of every ldmatrix
// come from eight different groups and hit eight different bank groups.  No
// host-encoded tensor map (no per-length encode, 256 sequences a launch),
// and nothing is read past a sequence's last position: the rows of a
// partial last tile that are not copied keep stale bytes, whose scores are
// masked and whose V elements are zeroed in the MMA fragments.
//
// Schedule.  With a static split of the tiles, per-SM streaming rates differ
// enough that the last CTA finishes ~40% after the median one.  Here each
// sequence is cut into chunks of C tiles (global chunk indices); CTA b
// starts on chunk b and claims chunk gridDim.x + (claim counter)++ each time
// it finishes issuing one, so fast SMs take more chunks.  Every chunk leaves
// per-warp partials (m, l, o) in its own workspace slots, so the split
// points -- and the result, bit for bit -- do not depend on which SM took
// which chunk; launch_slot_merge combines the slots in order.  A sequence
// that is one chunk on one warp per head is written directly.
//
// Roles (warp specialisation, no CTA-wide barrier in the main loop): warp 8
// is the producer -- lane 0 claims chunks (one ahead, hiding the atomic's
// latency) and arms the ring's `full` barriers, lanes 0-15 issue the group
// copies -- over a 3-stage ring released through `empty` barriers; warps 0-7
// consume: warp w serves kv head w % n_kv and the m-tiles w / n_kv (mod
// 8 / n_kv) of every tile, as in decode_mma.cu, and writes its partials at
// the end of each chunk without waiting for the other warps.
#include <math.h>

#include "decode.cuh"
#include "mma_frag.cuh"

namespace bml {

namespace {

constexpr int kSmemBudget = 227 * 1024;
constexpr int kWarps = 8;                  // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;  // + the producer warp
constexpr int kStageK = 32768;  // K bytes of a full tile (V the same), as decode.cu
constexpr int kStages = 3;
constexpr float kRescaleThreshold = 8.0f;

template <int D, int G>
struct BCfg {
    static constexpr int NT = (2 * G + 7) / 8;  // n8 column tiles of S (4 heads each)
    static constexpr int KS = D / 16;           // k-steps of S, d-blocks of O^T
    static constexpr int MTW = 128 / D;         // m-tiles per warp per tile
    static constexpr int SCR = 256;             // barriers, abort flag, stage info
};

// Bytes of one K (or V) tile of T rows: eight groups at pitch
// (T/8)*row_bytes + 16 (row_bytes is a multiple of 128).
__host__ __device__ __forceinline__ uint32_t ktile_bytes_of(uint32_t T, uint32_t row_bytes) {
    return T * row_bytes + 128u;
}

template <int D, int G>
uint32_t smem_bytes(uint32_t T, uint32_t row_bytes) {
    return kStages * 2u * ktile_bytes_of(T, row_bytes) + BCfg<D, G>::SCR + 128u;
}

// Sequence of global chunk c (binary search over the chunk ranges).
__device__ __forceinline__ uint32_t seq_of_chunk(const DecodeParams &p, uint32_t c) {
    uint32_t lo = 0, hi = p.n_seqs - 1;
    while (lo < hi) {
        const uint32_t mid = (lo + hi + 1) >> 1;
        if (p.seqs[mid].tile_begin <= c) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// What a filled ring stage holds, written by the producer before it arms
// the stage's barrier and read by the consumers after their wait.
struct StageInfo {
    uint32_t seq, row0, rows, chunk, flags;
};
constexpr uint32_t kFirstOfChunk = 1u, kLastOfChunk = 2u, kEnd = 4u;

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
    uint64_t *full = reinterpret_cast<uint64_t *>(scr);        // [kStages]
    uint64_t *empty = full + 4;                                // [kStages]
    volatile uint32_t *flags = reinterpret_cast<volatile uint32_t *>(full + 8);  // [0]: abort
    volatile StageInfo *info = reinterpret_cast<volatile StageInfo *>(full + 10);  // [kStages]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t CH = p.chunk_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kWarps);
        }
        flags[0] = 0u;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kWarps) {
        // ------------------------------------------------------- producer
        // Lane 0 walks the chunks: (chunk, sequence, first tile of the chunk
        // in the sequence, tiles in the chunk, tile within the chunk), with
        // the next chunk claimed when the current one starts.
        uint32_t ch = blockIdx.x, s = 0, first = 0, n = 0, j = 0, next = 0;
        bool done = false;
        auto start_chunk = [&]() {  // lane 0
            if (ch >= p.total_chunks) {
                done = true;
                return;
            }
            s = seq_of_chunk(p, ch);
            const DecodeSeq &sq = p.seqs[s];
            first = (ch - sq.tile_begin) * CH;
            n = min(CH, (sq.len + T - 1) / T - first);
            j = 0;
            next = gridDim.x + atomicAdd(&p.sched[0], 1u);
        };
        if (lane == 0) start_chunk();
        const uint64_t pol = l2_policy_evict_first();
        for (uint32_t it = 0;; ++it) {
            const uint32_t stage = it % kStages;
            bool ok = true;
            if (it >= (uint32_t)kStages) ok = mbar_wait(&empty[stage], ((it / kStages) - 1u) & 1u, flags, p.err);
            if (!__all_sync(0xffffffffu, ok)) break;
            uint32_t row0 = 0, rows = 0, seq = 0, end = 0;
            if (lane == 0) {
                if (done) {  // no more chunks: the consumers stop at this stage
                    info[stage].flags = kEnd;
                    mbar_arrive(&full[stage]);
                    end = 1u;
                } else {
                    const DecodeSeq &sq = p.seqs[s];
                    seq = s;
                    row0 = (first + j) * T;
                    rows = min(T, sq.len - row0);
                    info[stage].seq = s;
                    info[stage].row0 = row0;
                    info[stage].rows = rows;
                    info[stage].chunk = ch;
                    info[stage].flags = (j == 0 ? kFirstOfChunk : 0u) | (j + 1 == n ? kLastOfChunk : 0u);
                    mbar_arrive_expect_tx(&full[stage], 2u * rows * row_bytes);
                    if (++j == n) {
                        ch = next;
                        start_chunk();
                    }
                }
            }
            end = __shfl_sync(0xffffffffu, end, 0);
            if (end) break;
            seq = __shfl_sync(0xffffffffu, seq, 0);
            row0 = __shfl_sync(0xffffffffu, row0, 0);
            rows = __shfl_sync(0xffffffffu, rows, 0);
            __syncwarp();  // expected bytes are posted before any copy can complete
            // the consumers' generic-proxy reads of this stage (ordered by
            // the empty barrier) precede the async-proxy writes
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (lane < 16) {
                const uint32_t g8 = lane & 7u;  // group
                const uint32_t cnt = rows > g8 * gc ? min(gc, rows - g8 * gc) : 0u;
                if (cnt) {
                    const DecodeSeq &sq = p.seqs[seq];
                    const uint8_t *src = static_cast<const uint8_t *>(lane < 8 ? sq.k : sq.v) +
                                         ((size_t)row0 + g8 * gc) * row_bytes;
                    bulk_g2s_stream(stages + stage * stage_bytes + (lane < 8 ? 0u : ktile_bytes) + g8 * gpitch, src,
                                    cnt * row_bytes, &full[stage], pol);
                }
            }
            __syncwarp();
        }
    } else {
        // ------------------------------------------------------- consumers
        const int g = lane >> 2, c = lane & 3;  // mma fragment row / column pair
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

        // byte offset of 16-byte chunk `chunk` (0 .. D/8-1) of this warp's
        // head at row r (0..15) of m-tile mt, i.e. position (r % 8) * gc +
        // 2*mt + r / 8
        const uint32_t head_off = (uint32_t)h * D * 2u;
        auto chunk_off = [&](uint32_t mt, uint32_t r, uint32_t chunk) {
            return (r & 7u) * gpitch + (2u * mt + (r >> 3)) * row_bytes + head_off + (chunk << 4);
        };
        auto pos_of = [&](uint32_t mt, uint32_t r) { return (r & 7u) * gc + 2u * mt + (r >> 3); };

        uint32_t s = 0;
        bool fresh = true;  // no tile of the current chunk processed yet
        for (uint32_t it = 0;; ++it) {
            const uint32_t stage = it % kStages;
            const bool ok = mbar_wait(&full[stage], (it / kStages) & 1u, flags, p.err);
            if (!__all_sync(0xffffffffu, ok)) break;  // timed out: leave (no barrier waits for us)
            const uint32_t sflags = info[stage].flags;
            if (sflags & kEnd) break;
            const uint32_t row0 = info[stage].row0;
            const uint32_t rows = info[stage].rows;
            const uint32_t chunk = info[stage].chunk;
            if (sflags & kFirstOfChunk) {  // every chunk is its own partial
                s = info[stage].seq;
                load_q(s);
                fresh = true;
            }
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

            __syncwarp();  // the warp's shared-memory reads of the stage precede the release
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (!(sflags & kLastOfChunk)) continue;

            // ------------- this warp's partial of the chunk: (m, l, o / l) of
            // its G heads over its m-tiles, into slot chunk * nph + ph (or
            // straight to the output for a one-slot sequence)
            const DecodeSeq &sq = p.seqs[s];
            const uint32_t slot = sq.slot_base + (chunk - sq.tile_begin) * (uint32_t)nph + (uint32_t)ph;
            const bool single = sq.n_slots == 1;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float L = l_part[nt];
                L += __shfl_xor_sync(0xffffffffu, L, 4);
                L += __shfl_xor_sync(0xffffffffu, L, 8);
                L += __shfl_xor_sync(0xffffffffu, L, 16);
                const int hd = nt * 4 + c;
                if (hd < G) {
                    const uint32_t qh = (uint32_t)h * G + hd;
                    const float inv = L > 0.f ? 1.f / L : 0.f;  // a warp with no valid row writes zeros
                    const size_t row = (size_t)s * p.n_heads + qh;
                    const size_t srow = (size_t)slot * p.n_heads + qh;
                    float *dst = single ? (p.mode == kModeFinal ? p.out : p.part_o) + row * D
                                        : p.slot_o + srow * D;
#pragma unroll
                    for (int db = 0; db < KS; ++db) {
                        dst[db * 16 + g] = (o[nt][db][0] + o[nt][db][1]) * inv;
                        dst[db * 16 + g + 8] = (o[nt][db][2] + o[nt][db][3]) * inv;
                    }
                    if (g == 0) {
                        if (!single) {
                            p.slot_ml[srow * 2 + 0] = m_run[nt];
                            p.slot_ml[srow * 2 + 1] = L;
                        } else if (p.mode != kModeFinal) {
                            p.part_m[row] = m_run[nt];
                            p.part_l[row] = L;
                        }
                    }
                }
            }
        }
    }

    // The last CTA to leave resets the claim counter for the next call.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&p.sched[1], 1u) == gridDim.x - 1) {
            p.sched[0] = 0u;
            p.sched[1] = 0u;
            __threadfence();
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
    if (p.rows_per_tile * p.row_bytes > (uint32_t)kStageK || p.row_bytes % 128 != 0 || p.rows_per_tile % 16 != 0)
        return cudaErrorInvalidValue;
    // dynamic schedule only: every CTA starts on chunk blockIdx.x
    if (p.chunk_tiles == 0 || !p.sched || grid <= 0 || (uint32_t)grid > p.total_chunks) return cudaErrorInvalidValue;
    const bool f16 = dt == BML_F16;
    if (head_dim == 128) return f16 ? launch_g<128, true>(p, group, grid, stream) : launch_g<128, false>(p, group, grid, stream);
    return f16 ? launch_g<64, true>(p, group, grid, stream) : launch_g<64, false>(p, group, grid, stream);
}

}  // namespace bml
