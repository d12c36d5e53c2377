// decode_bulk.cu -- split-K flash decoding for 16-bit KV caches: group bulk
// copies + warp-level tensor-core MMAs, tiles claimed at run time, partials
// merged in the same launch (sm_100a).
//
// Computes, for every sequence of a batch, the attention block of
// forward_layer_cached (crates/compiler/src/gguf_compiler.rs:1008-1050 in
// SugarFreeDoNoSo/bml): scores q.k * scale over every cached position, a
// max-subtracted softmax and the P.V sum for the n_heads / n_kv q heads that
// share each kv head.  m16n8k16 MMAs take q and P as exact pairs of 16-bit
// terms, so products are exact and sums f32 (within 1e-4 of the reference's
// f32 / f64 arithmetic).
//
// Loads.  A tile of T positions of a cache ([len][n_kv][D], row_bytes =
// n_kv*D*2 contiguous bytes per position) arrives as eight 1-D bulk copies,
// one per group of Gc = T/8 consecutive positions, each group landing 16
// bytes further along modulo 128 than the one before (group pitch
// Gc*row_bytes + 16).  The MMA row order inside a 16-position m-tile is free
// (the softmax and P.V only need to agree on it), so m-tile mt's row r is
// position (r % 8) * Gc + 2*mt + r / 8: the eight rows of every ldmatrix
// come from eight different groups and hit eight different bank groups.
// Nothing is read past a sequence's last position: the rows of a partial
// last tile that are not copied keep stale bytes, whose scores are masked
// and whose V elements are zeroed in the MMA fragments.
//
// Schedule.  Per-SM streaming rates differ enough that a static split of
// the tiles leaves the last CTA finishing ~40% after the median one, and a
// partial per fixed-size chunk costs either balance (large chunks) or
// partial traffic and a separate merge launch (small ones).  Here:
//  * the host deals the CTAs to the sequences as home CTAs (fewest tiles per
//    home CTA at worst, decode_assign_homes); the home CTAs of a sequence
//    take its first tiles and its first parts statically, one each, so every
//    CTA issues its first copy without waiting on an atomic;
//    further tiles are claimed claim_tiles at a time from a per-sequence
//    counter (the producer claims one claim ahead, hiding the atomic);
//  * a CTA carries its running (m, l, o) over every tile it takes of a
//    sequence (its "visit"); when the sequence has no unclaimed tile left it
//    writes that carry as one part and moves to the sequence with the most
//    unclaimed tiles, so every CTA works to the end and the tail is about
//    one claim;
//  * a joining visit first reserves one of the sequence's parts_per_seq part
//    slots; a sequence that has them all taken has that many CTAs still on
//    it, so every tile is processed by some running CTA (no CTA ever waits on
//    one that has not started);
//  * reservations and the done count of a sequence share one 64-bit word,
//    so one load tells both whether the sequence is complete and how many
//    parts it has;
//  * when no tile is left to claim, the producer claims a merge item (a
//    block of q-head rows of one sequence) and waits (bounded) until its
//    sequence is complete while the consumers drain the ring; the consumers
//    then combine that sequence's parts with the log-sum-exp rule, write
//    the output, and claim further items one ahead.
// Parts of a sequence depend on which CTA took which tile, so results agree
// with the reference to the decode tolerance but may differ between runs in
// the last bits.
//
// Roles (warp specialisation): warp NW is the producer -- lane 0 claims
// tiles and reserves parts, the warp picks the next sequence (one counter
// per lane), lanes 0-15 issue the group copies -- over a 3-stage ring whose
// stages are tiles or control records (visit start, flush, end), released
// through `empty` barriers; warps 0..NW-1 consume (NW = 8 for head_dim 128,
// 16 for 64): warp w serves kv head w % n_kv and the m-tiles w / n_kv (mod
// NW / n_kv) of every tile, and at a flush writes its own partial for its
// heads (NW / n_kv partial slots a part) with no CTA-wide barrier.
#include <math.h>

#include <algorithm>

#include "decode.cuh"
#include "mma_frag.cuh"

namespace bml {

namespace {

constexpr int kSmemBudget = 227 * 1024;
constexpr int kStageK = 32768;               // K bytes of a full tile (V the same)
constexpr int kStages = 3;
constexpr float kRescaleThreshold = 8.0f;
constexpr unsigned kFull = 0xffffffffu;
constexpr uint32_t kNone = 0xffffffffu;

// NW consumer warps (decode_bulk_warps: 8 for head_dim 128, 16 for 64) + one
// producer warp.
template <int D, int G, int NW>
struct BCfg {
    static constexpr int THREADS = (NW + 1) * 32;
    static constexpr int NT = (2 * G + 7) / 8;  // n8 column tiles of S (4 heads each)
    static constexpr int KS = D / 16;           // k-steps of S, d-blocks of O^T
    static constexpr int MTW = 1024 / (D * NW);  // m-tiles per warp per tile
    static constexpr int SCR = 256;             // barriers, flags, stage records
    static constexpr int MERGE = NW * (D + 4) * 4;  // merge scratch: per warp (M, L, -, -, O[D])
    static_assert(MTW >= 1, "at most one warp per m-tile");
};

// Bytes of one K (or V) tile of T rows: eight groups at pitch
// (T/8)*row_bytes + 16 (row_bytes is a multiple of 128).
__host__ __device__ __forceinline__ uint32_t ktile_bytes_of(uint32_t T, uint32_t row_bytes) {
    return T * row_bytes + 128u;
}

template <int D, int G, int NW>
uint32_t smem_bytes(uint32_t T, uint32_t row_bytes) {
    // the merge stages its slots in the ring: every warp's batch fits in it
    static_assert(NW * 32u * (D + 3u) * 4u <= kStages * 2u * 32768u, "merge staging exceeds the ring");
    return kStages * 2u * ktile_bytes_of(T, row_bytes) + BCfg<D, G, NW>::SCR + BCfg<D, G, NW>::MERGE + 128u;
}

__device__ __forceinline__ uint32_t tiles_of(const DecodeParams &p, uint32_t s) {
    return (p.seqs[s].len + p.rows_per_tile - 1) / p.rows_per_tile;
}

// Home CTAs of sequence s (decode_assign_homes): they hold its first tiles
// and parts.
__device__ __forceinline__ uint32_t homes_of(const DecodeParams &p, uint32_t s) { return p.seqs[s].n_slots; }

// The home sequence of CTA b: the last sequence whose first home CTA is at
// or before b (sequences without homes share the next one's first CTA).
__device__ __forceinline__ uint32_t home_of_cta(const DecodeParams &p, uint32_t b) {
    uint32_t lo = 0, hi = p.n_seqs - 1;
    while (lo < hi) {
        const uint32_t mid = (lo + hi + 1) >> 1;
        if (p.seqs[mid].slot_base <= b) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

constexpr uint32_t kNoItem = 0xffffffffu;

__device__ __forceinline__ void st_release_gpu(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread: claims the next merge item -- item i belongs to the (i /
// ips)-th sequence to complete, and is block i % ips of its (row block,
// head-dim slice) pieces -- and waits (bounded by p.wait_ns) until that
// sequence is in the completion queue.  Returns false when every item is
// taken, the wait gave up or the CTA is aborting; else sets item, seq and
// np, the sequence's number of parts (home parts + joiners' reservations, at
// most parts_per_seq).
__device__ __noinline__ bool claim_item(const DecodeParams &p, const unsigned long long *state,
                                           const uint32_t *queue, uint32_t ips, uint32_t items,
                                           volatile uint32_t *abort_flag, uint32_t &item, uint32_t &seq,
                                           uint32_t &np) {
    if (*abort_flag) return false;
    item = atomicAdd(&p.sched[1], 1u);
    if (item >= items) return false;
    uint64_t t0 = 0;
    for (uint32_t polls = 0;; ++polls) {
        const uint32_t v = ld_acquire_gpu(&queue[item / ips]);
        if (v) {
            seq = v - 1u;
            break;
        }
        if (*abort_flag) return false;
        const uint64_t now = globaltimer_ns();
        if (!t0) t0 = now;
        if (now - t0 > p.wait_ns) {
            *abort_flag = 1u;
            atomicOr(p.err, kErrTimeout);
            return false;
        }
        if (polls > 8) __nanosleep(64);
    }
    const unsigned long long st = ld_acquire_gpu_u64(&state[seq]);
    np = min(homes_of(p, seq) + (uint32_t)(st >> 32), p.parts_per_seq);
    return true;
}

template <int BYTES>
__device__ __forceinline__ void cp_async(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(smem_u32(dst)), "l"(src), "n"(BYTES)
                 : "memory");
}

// Shared-memory bytes one consumer warp stages per batch of merge slots.
template <int D>
__host__ __device__ constexpr uint32_t merge_stage_bytes() {
    return 32u * (D + 3u) * 4u;
}

// This warp's share of the partial slots of RW q-head rows (qh[i]) of
// sequence sq, for VS head dims per lane starting at dim0: slots j = sub,
// sub + wpr, ... of the nsub = parts * nph slots, combined with the
// log-sum-exp rule into (M, L, O) relative to M.  A batch of up to 32 / RW
// slots per row is staged in the warp's shared memory with cp.async first
// (lane u also copies slot u's (m, l) and tile count), so all of its loads
// are in flight at once and take no registers.  Empty parts (0 tiles) and
// slots of warps that saw no valid row (m = -inf) are skipped by selection,
// never multiplied (their bytes may be stale).
template <int D, int VS, int RW>
__device__ __forceinline__ void merge_share(const DecodeParams &p, uint32_t sq, const uint32_t (&qh)[RW],
                                            uint32_t dim0, uint32_t nsub, uint32_t nph, uint32_t sub, uint32_t wpr,
                                            int lane, uint8_t *wstage, float (&M)[RW], float (&L)[RW],
                                            float (&O)[RW][VS]) {
    constexpr int UN = 32 / RW;
    constexpr float NEG_INF = -INFINITY;
    // staging: o [RW][UN][32 * VS] | (m, l) [RW][UN] | tiles [RW][UN]
    float *so = reinterpret_cast<float *>(wstage);
    float2 *sml = reinterpret_cast<float2 *>(so + RW * UN * 32 * VS);
    uint32_t *stl = reinterpret_cast<uint32_t *>(sml + RW * UN);
#pragma unroll
    for (int i = 0; i < RW; ++i) {
        M[i] = NEG_INF;
        L[i] = 0.f;
#pragma unroll
        for (int e = 0; e < VS; ++e) O[i][e] = 0.f;
    }
    for (uint32_t j0 = sub; j0 < nsub; j0 += (uint32_t)UN * wpr) {
        const uint32_t nb = min((uint32_t)UN, (nsub - j0 + wpr - 1) / wpr);  // slots of this batch
#pragma unroll
        for (int i = 0; i < RW; ++i) {
            for (uint32_t u = 0; u < nb; ++u) {
                const uint32_t jj = j0 + u * wpr;
                const uint32_t prt = sq * p.parts_per_seq + jj / nph;
                const size_t srow = ((size_t)prt * nph + jj % nph) * p.n_heads + qh[i];
                cp_async<VS * 4>(so + ((size_t)i * UN + u) * 32 * VS + lane * VS,
                                 p.slot_o + srow * D + dim0 + lane * VS);
            }
            if ((uint32_t)lane < nb) {
                const uint32_t jj = j0 + (uint32_t)lane * wpr;
                const uint32_t prt = sq * p.parts_per_seq + jj / nph;
                const size_t srow = ((size_t)prt * nph + jj % nph) * p.n_heads + qh[i];
                cp_async<8>(sml + i * UN + lane, p.slot_ml + srow * 2);
                cp_async<4>(stl + i * UN + lane, p.part_tiles + prt);
            }
        }
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
        __syncwarp();  // every lane's copies are visible to the whole warp
#pragma unroll
        for (int i = 0; i < RW; ++i) {
            for (uint32_t u = 0; u < nb; ++u) {
                const float2 ml = sml[i * UN + u];
                if (stl[i * UN + u] == 0u || ml.x == NEG_INF) continue;
                const float Mn = fmaxf(M[i], ml.x);
                const float a = M[i] == NEG_INF ? 0.f : fast_exp2(M[i] - Mn);
                const float b = fast_exp2(ml.x - Mn) * ml.y;
                L[i] = L[i] * a + b;
                const float *ov = so + ((size_t)i * UN + u) * 32 * VS + lane * VS;
#pragma unroll
                for (int e = 0; e < VS; ++e) O[i][e] = O[i][e] * a + ov[e] * b;
                M[i] = Mn;
            }
        }
        __syncwarp();  // the batch is read before the next one lands
    }
}

// Writes dims [dim0 + lane * VS, + VS) of merged row `row` (sequence-major)
// from (M, L, O): the output O / L, and in partial mode (M, L) once per row.
template <int D, int VS>
__device__ __forceinline__ void merge_store(const DecodeParams &p, size_t row, uint32_t dim0, float M, float L,
                                            const float (&O)[VS], int lane) {
    const float inv = L > 0.f ? 1.f / L : 0.f;
    float *dst = (p.mode == kModeFinal ? p.out : p.part_o) + row * D + dim0 + lane * VS;
#pragma unroll
    for (int e = 0; e < VS; ++e) dst[e] = O[e] * inv;
    if (p.mode != kModeFinal && lane == 0 && dim0 == 0) {
        p.part_m[row] = M;
        p.part_l[row] = L;
    }
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One warp, one exchange unit (q-head row qh, dims [dim0, dim0 + 32)) of a
// KV split over GPUs.  This rank's (M, L, O / L) -- lane l holds dim l --
// goes to every rank's buffer slot [parity][this rank][unit] with plain
// stores over peer memory, then a release store of the call's epoch (the
// next value of this rank's device-side call counter) into that rank's flag
// for it.  Lane r waits (bounded by p.wait_ns) for rank
// r's flag in this rank's buffer; the ranks' units are then merged in rank
// order (so all ranks write bit-identical outputs).  A slot is reused two
// calls later: by then every rank has finished the call that read it (a
// rank's next call starts after its previous one, on one stream).
__device__ __noinline__ void exchange_store(const DecodeParams &p, uint32_t unit, uint32_t qh, uint32_t dim0,
                                            float M, float L, float O, int lane) {
    constexpr float NEG_INF = -INFINITY;
    // the counter changes only at the exit of this launch's last CTA, after
    // every exchange of the launch: all CTAs read the same value here
    const uint32_t epoch = exchange_next_epoch(__ldcg(p.x_epoch));
    const uint32_t par = epoch & 1u, W = p.x_world;
    const size_t data = exchange_data_floats(p.x_units);
    const size_t mine = ((size_t)(par * kMaxExchangeRanks + p.x_rank) * p.x_units + unit) * kExchangeUnitFloats;
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (uint32_t r = 0; r < W; ++r) {
        float *dst = p.x_base[r] + mine;
        if (lane == 0) {
            dst[0] = M;
            dst[1] = L;
        }
        dst[4 + lane] = O * inv;
    }
    __threadfence_system();  // the unit reaches every rank before its flag
    __syncwarp();
    const size_t fl = (size_t)(par * kMaxExchangeRanks + p.x_rank) * p.x_units + unit;
    if ((uint32_t)lane < W) st_release_sys(reinterpret_cast<uint32_t *>(p.x_base[lane] + data) + fl, epoch);
    bool ok = true;
    if ((uint32_t)lane < W) {
        const uint32_t *flag = reinterpret_cast<const uint32_t *>(p.x_base[p.x_rank] + data) +
                               (size_t)(par * kMaxExchangeRanks + lane) * p.x_units + unit;
        uint64_t t0 = 0;
        for (uint32_t polls = 0; ld_acquire_sys(flag) != epoch; ++polls) {
            const uint64_t now = globaltimer_ns();
            if (!t0) t0 = now;
            if (now - t0 > p.wait_ns) {
                atomicOr(p.err, kErrTimeout);
                ok = false;
                break;
            }
            if (polls > 8) __nanosleep(32);
        }
    }
    if (!__all_sync(0xffffffffu, ok)) return;  // the error word reports it
    const float *base = p.x_base[p.x_rank];
    float Mt = NEG_INF;
    for (uint32_t r = 0; r < W; ++r)
        Mt = fmaxf(Mt, __ldcv(base + ((size_t)(par * kMaxExchangeRanks + r) * p.x_units + unit) * kExchangeUnitFloats));
    float Lt = 0.f, Ot = 0.f;
    for (uint32_t r = 0; r < W; ++r) {
        const float *u = base + ((size_t)(par * kMaxExchangeRanks + r) * p.x_units + unit) * kExchangeUnitFloats;
        const float mr = __ldcv(u);
        const float w = mr == NEG_INF ? 0.f : fast_exp2(mr - Mt) * __ldcv(u + 1);
        Lt += w;
        Ot += __ldcv(u + 4 + lane) * w;
    }
    p.out[(size_t)qh * 32u * (p.x_units / p.n_heads) + dim0 + lane] = Lt > 0.f ? Ot / Lt : 0.f;
}

// The consumer warps' merge of one item: R q-head rows starting at row0 of
// sequence sq, head dims [dim0, dim0 + 32 * VS).  wpr warps share a row
// (warp w takes row w / wpr and the slots w % wpr (mod wpr); their running
// (M, L, O) are combined in warp order through shared memory), or, with RW
// = 2, each warp takes two rows.  Every consumer thread calls it (the
// combine has a named barrier).  `stage` is the ring's shared memory, idle
// once the stream has ended.  Not inlined, so that it takes no registers
// from the streaming loop.
template <int D, int VS, int RW, int NW>
__device__ __noinline__ void merge_item(const DecodeParams &p, uint32_t sq, uint32_t row0, uint32_t dim0,
                                           uint32_t nsub, uint32_t nph, uint32_t wpr, int warp, int lane,
                                           float *mscr, uint8_t *stage) {
    constexpr float NEG_INF = -INFINITY;
    const uint32_t sub = (uint32_t)warp % wpr;
    uint32_t qh[RW];
#pragma unroll
    for (int i = 0; i < RW; ++i) qh[i] = RW == 2 ? row0 + (uint32_t)warp * 2u + i : row0 + (uint32_t)warp / wpr;
    float M[RW], L[RW], O[RW][VS];
    merge_share<D, VS, RW>(p, sq, qh, dim0, nsub, nph, RW == 2 ? 0u : sub, RW == 2 ? 1u : wpr, lane,
                           stage + (size_t)warp * merge_stage_bytes<D>(), M, L, O);
    if (RW == 1 && wpr > 1) {
        float *mine = mscr + warp * (D + 4);
        if (lane == 0) {
            mine[0] = M[0];
            mine[1] = L[0];
        }
#pragma unroll
        for (int e = 0; e < VS; ++e) mine[4 + lane * VS + e] = O[0][e];
        named_bar_sync(1, NW * 32);
        if (sub == 0) {
            float Mt = NEG_INF;
            for (uint32_t i = 0; i < wpr; ++i) Mt = fmaxf(Mt, mscr[(warp + i) * (D + 4)]);
            L[0] = 0.f;
#pragma unroll
            for (int e = 0; e < VS; ++e) O[0][e] = 0.f;
            for (uint32_t i = 0; i < wpr; ++i) {
                const float *w = mscr + (warp + i) * (D + 4);
                const float f = w[0] == NEG_INF ? 0.f : fast_exp2(w[0] - Mt);
                L[0] += w[1] * f;
#pragma unroll
                for (int e = 0; e < VS; ++e) O[0][e] += w[4 + lane * VS + e] * f;
            }
            M[0] = Mt;
        }
    }
    if (RW == 1 && VS == 1 && p.x_world > 1) {
        if (sub == 0) exchange_store(p, qh[0] * (D / 32) + dim0 / 32, qh[0], dim0, M[0], L[0], O[0][0], lane);
    } else if (RW == 2 || sub == 0) {
#pragma unroll
        for (int i = 0; i < RW; ++i)
            merge_store<D, VS>(p, (size_t)sq * p.n_heads + qh[i], dim0, M[i], L[i], O[i], lane);
    }
}

// Ring stage records, written by the producer before it arms the stage and
// read by the consumers after their wait.
struct StageInfo {
    uint32_t kind, seq, row0, rows, part, tiles;
};
constexpr uint32_t kTile = 0u, kVisit = 1u, kFlush = 2u, kEnd = 3u;

// ----------------------------------------------------------------- kernel
template <int D, int G, bool F16, int NW>
__global__ void __launch_bounds__(BCfg<D, G, NW>::THREADS, 1)
    decode_bulk_kernel(const __grid_constant__ DecodeParams p) {
    using C = BCfg<D, G, NW>;
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
    // [0] abort, [1] merge item, [2] merge parts, [3] last CTA to leave
    volatile uint32_t *flags = reinterpret_cast<volatile uint32_t *>(full + 8);
    volatile StageInfo *info = reinterpret_cast<volatile StageInfo *>(full + 12);  // [kStages]
    float *mscr = reinterpret_cast<float *>(scr + C::SCR);    // [NW][D + 4]

    // per sequence: tiles claimed past the home tiles, and a state word whose
    // high half counts joining visits' part reservations and low half the
    // tiles done (8 per tile, one per consumer warp)
    uint32_t *const claim_c = p.counters;
    unsigned long long *const state = reinterpret_cast<unsigned long long *>(p.counters + kMaxSeqsPerLaunch);
    uint32_t *const queue = p.counters + 3 * kMaxSeqsPerLaunch;  // completed sequences + 1, in order
    uint32_t *const left_c = p.counters + 4 * kMaxSeqsPerLaunch;  // visits that ended

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t nph = NW / p.n_kv;  // warps per kv head = partial slots per part
    const uint32_t U = p.claim_tiles;
    const uint32_t R = p.merge_rows, wpr = p.merge_wpr, DS = p.merge_dsplit;
    const uint32_t ips = p.n_heads / R * DS;  // merge items per sequence
    const uint32_t items = p.n_seqs * ips;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NW);
        }
        flags[0] = 0u;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NW) {
        // ------------------------------------------------------- producer
        const uint64_t pol = l2_policy_evict_first();
        uint32_t it = 0;  // stages posted
        // the next ring stage, once its consumers released it; false on timeout
        auto acquire = [&](uint32_t &stage) -> bool {
            stage = it % kStages;
            bool ok = true;
            if (it >= (uint32_t)kStages)
                ok = mbar_wait(&empty[stage], ((it / kStages) - 1u) & 1u, flags, p.err, p.wait_ns);
            return __all_sync(kFull, ok);
        };
        // a stage without data: a visit start, a flush or the end
        auto post_ctl = [&](uint32_t kind, uint32_t seq, uint32_t part, uint32_t tiles) -> bool {
            uint32_t stage;
            if (!acquire(stage)) return false;
            if (lane == 0) {
                info[stage].kind = kind;
                info[stage].seq = seq;
                info[stage].part = part;
                info[stage].tiles = tiles;
                mbar_arrive(&full[stage]);
            }
            ++it;
            __syncwarp();
            return true;
        };
        // The end record carries the CTA's first merge item, its sequence and
        // part count, claimed and waited for here while the consumers drain
        // the ring.
        auto post_end = [&]() {
            uint32_t item = kNoItem, seq = 0, np = 0;
            if (lane == 0 && !claim_item(p, state, queue, ips, items, flags, item, seq, np)) item = kNoItem;
            item = __shfl_sync(kFull, item, 0);
            seq = __shfl_sync(kFull, seq, 0);
            np = __shfl_sync(kFull, np, 0);
            post_ctl(kEnd, item, np, seq);
        };
        // Warp: the sequence where a joining CTA helps most -- the most
        // unclaimed tiles per CTA already on it (reserved parts minus ended
        // visits), lowest index on ties -- among those with a part left and,
        // unless no CTA is on it yet, at least join_min unclaimed tiles per
        // CTA on it (a smaller remainder is finished by those CTAs sooner
        // than a join takes); kNone if there is none.  A sequence with
        // unclaimed tiles has every CTA that took a part of it still on it,
        // so the rule leaves no tile behind.  The counters only grow, so a
        // stale read never hides remaining work.
        auto pick = [&]() -> uint32_t {
            uint32_t cl[kMaxSeqsPerLaunch / 32], rs[kMaxSeqsPerLaunch / 32], lf[kMaxSeqsPerLaunch / 32];
#pragma unroll
            for (int i = 0; i < kMaxSeqsPerLaunch / 32; ++i) {
                const uint32_t s = (uint32_t)i * 32u + (uint32_t)lane;
                cl[i] = rs[i] = lf[i] = 0u;
                if (s < p.n_seqs) {
                    cl[i] = ld_relaxed_gpu(&claim_c[s]);
                    rs[i] = (uint32_t)(ld_relaxed_gpu_u64(&state[s]) >> 32);
                    lf[i] = ld_relaxed_gpu(&left_c[s]);
                }
            }
            uint32_t best = kNone, best_score = 0;
#pragma unroll
            for (int i = 0; i < kMaxSeqsPerLaunch / 32; ++i) {
                if ((uint32_t)i * 32u >= p.n_seqs) break;
                const uint32_t s = (uint32_t)i * 32u + (uint32_t)lane;
                uint32_t score = 0;  // unclaimed tiles per CTA on it, scaled by 16; 0 = not worth joining
                if (s < p.n_seqs) {
                    const uint32_t nt = tiles_of(p, s), h = homes_of(p, s);
                    const uint32_t claimed = h + cl[i], taken = h + rs[i];
                    if (claimed < nt && taken < p.parts_per_seq) {
                        const uint32_t rem = nt - claimed;
                        const uint32_t on = taken > lf[i] ? taken - lf[i] : 0u;
                        if (on == 0 || rem >= p.join_min * on) score = (16u * rem) / (on + 1u) + 1u;
                    }
                }
                const uint32_t mx = __reduce_max_sync(kFull, score);
                if (mx > best_score) {
                    best_score = mx;
                    best = (uint32_t)i * 32u + (uint32_t)(__ffs(__ballot_sync(kFull, score == mx)) - 1);
                }
            }
            return best;
        };

        // visit state (lane 0's copy is the authoritative one): sequence s,
        // part, current claim [c, c + cn), next tile j of it, tiles of the
        // visit so far vt, prefetched next claim pref
        uint32_t s = 0, part = 0, c = 0, cn = 0, j = 0, vt = 0, pref = 0;

        // Warp: opens a joining visit on the best pick and posts its visit
        // record; false if no tile is left anywhere (or on timeout).
        auto join = [&]() -> bool {
            for (uint32_t tries = 0; tries <= 2u * p.n_seqs + 2u; ++tries) {
                const uint32_t cand = pick();
                if (cand == kNone) return false;
                uint32_t ok = 0;
                if (lane == 0) {
                    const uint32_t h = homes_of(p, cand), nt = tiles_of(p, cand);
                    const uint32_t k = h + (uint32_t)(atomicAdd(&state[cand], 1ull << 32) >> 32);
                    if (k < p.parts_per_seq) {
                        const uint32_t cc = h + atomicAdd(&claim_c[cand], U);
                        if (cc < nt) {  // else an empty part: its tile count stays 0
                            ok = 1u;
                            s = cand;
                            part = cand * p.parts_per_seq + k;
                            c = cc;
                            cn = min(U, nt - c);
                            j = 0;
                            vt = 0;
                            pref = h + atomicAdd(&claim_c[s], U);  // the next claim, one ahead
                        }
                    }
                }
                if (__shfl_sync(kFull, ok, 0)) {
                    const uint32_t ss = __shfl_sync(kFull, s, 0), pp = __shfl_sync(kFull, part, 0);
                    return post_ctl(kVisit, ss, pp, 0u);
                }
            }
            return false;
        };

        bool run = (p.diag & kDiagStall) == 0u;
        if (run) {
            // the home visit: first tile and part by rank among the home CTAs
            const uint32_t home = home_of_cta(p, blockIdx.x);
            const uint32_t r = blockIdx.x - p.seqs[home].slot_base;
            s = home;
            part = home * p.parts_per_seq + r;
            c = r;
            cn = 1;
            j = 0;
            vt = 0;
            if (lane == 0) pref = homes_of(p, s) + atomicAdd(&claim_c[s], U);
            run = post_ctl(kVisit, s, part, 0u);
        }
        while (run) {
            uint32_t stage;
            if (!acquire(stage)) break;
            uint32_t row0 = 0, rows = 0, seq = 0, flush = 0;
            if (lane == 0) {
                const DecodeSeq &sq = p.seqs[s];
                seq = s;
                row0 = (c + j) * T;
                rows = min(T, sq.len - row0);
                info[stage].kind = kTile;
                info[stage].seq = s;
                info[stage].row0 = row0;
                info[stage].rows = rows;
                mbar_arrive_expect_tx(&full[stage], 2u * rows * row_bytes);
            }
            ++it;
            seq = __shfl_sync(kFull, seq, 0);
            row0 = __shfl_sync(kFull, row0, 0);
            rows = __shfl_sync(kFull, rows, 0);
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
            // the claim bookkeeping (which may wait on the prefetched claim)
            // comes after the copies are on their way
            if (lane == 0) {
                ++j;
                ++vt;
                if (j == cn) {  // claim used up: the prefetched one, or the visit ends
                    const uint32_t nt = tiles_of(p, s);
                    if (pref < nt) {
                        c = pref;
                        cn = min(U, nt - c);
                        j = 0;
                        pref = homes_of(p, s) + atomicAdd(&claim_c[s], U);
                    } else {
                        flush = 1u;
                    }
                }
            }
            flush = __shfl_sync(kFull, flush, 0);
            if (flush) {
                if (lane == 0) atomicAdd(&left_c[s], 1u);  // this CTA leaves the sequence
                const uint32_t ss = __shfl_sync(kFull, s, 0), pp = __shfl_sync(kFull, part, 0);
                const uint32_t tt = __shfl_sync(kFull, vt, 0);
                if (!post_ctl(kFlush, ss, pp, tt)) break;
                if (!join()) {
                    if (!__shfl_sync(kFull, flags[0], 0)) post_end();  // uniform: post_end is collective
                    break;
                }
            }
        }
        // After a timeout, copies of the last stages may still be landing in
        // shared memory: wait (bounded) for them before the CTA leaves.
        if (flags[0] && lane == 0) {
            for (uint32_t pos = it > (uint32_t)kStages ? it - kStages : 0u; pos < it; ++pos)
                mbar_drain(&full[pos % kStages], (pos / kStages) & 1u, p.wait_ns);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------- consumers
        const int g = lane >> 2, c = lane & 3;  // mma fragment row / column pair
        const int n_kv = (int)p.n_kv;
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

        // This warp's partial of the visit -- (m, l, o / l) of its G heads
        // over its m-tiles -- into slot part * nph + ph; then its share of
        // the sequence's done count.  A warp with no valid row writes m =
        // -inf, l = 0 and zeros, never 0/0.
        auto flush = [&](uint32_t seq, uint32_t prt, uint32_t tiles) {
            const size_t sub = (size_t)prt * nph + (uint32_t)ph;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float L = l_part[nt];
                L += __shfl_xor_sync(kFull, L, 4);
                L += __shfl_xor_sync(kFull, L, 8);
                L += __shfl_xor_sync(kFull, L, 16);
                const int hd = nt * 4 + c;
                if (hd < G) {
                    const uint32_t qh = (uint32_t)h * G + hd;
                    const float inv = L > 0.f ? 1.f / L : 0.f;
                    const size_t srow = sub * p.n_heads + qh;
                    float *dst = p.slot_o + srow * D;
#pragma unroll
                    for (int db = 0; db < KS; ++db) {
                        dst[db * 16 + g] = (o[nt][db][0] + o[nt][db][1]) * inv;
                        dst[db * 16 + g + 8] = (o[nt][db][2] + o[nt][db][3]) * inv;
                    }
                    if (g == 0) *reinterpret_cast<float2 *>(p.slot_ml + srow * 2) = make_float2(m_run[nt], L);
                }
            }
            if (lane == 0) p.part_tiles[prt] = tiles;
            __threadfence();  // the partial is visible before the done count moves
            __syncwarp();
            if (lane == 0) {
                // the warp whose count completes the sequence queues it for
                // the merge
                const unsigned long long old = atomicAdd(&state[seq], (unsigned long long)tiles);
                if ((uint32_t)old + tiles == (uint32_t)NW * tiles_of(p, seq))
                    st_release_gpu(&queue[atomicAdd(&p.sched[2], 1u)], seq + 1u);
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

        uint32_t s = 0, part = 0;
        uint32_t end_item = kNoItem, end_np = 0, end_seq = 0;
        bool fresh = true;  // no tile of the current visit processed yet
        for (uint32_t it = 0;; ++it) {
            const uint32_t stage = it % kStages;
            const bool ok = mbar_wait(&full[stage], (it / kStages) & 1u, flags, p.err, p.wait_ns);
            if (!__all_sync(kFull, ok)) break;  // timed out: leave (no barrier waits for us)
            const uint32_t kind = info[stage].kind;
            if (kind != kTile) {
                const uint32_t iseq = info[stage].seq, ipart = info[stage].part, itiles = info[stage].tiles;
                if (kind == kEnd) {  // no release: nothing is posted after it
                    end_item = iseq;
                    end_np = ipart;
                    end_seq = itiles;
                    break;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[stage]);
                if (kind == kVisit) {
                    s = iseq;
                    part = ipart;
                    load_q(s);
                    fresh = true;
                } else {
                    flush(s, part, itiles);
                }
                continue;
            }
            const uint32_t rows = info[stage].rows;
            const uint32_t sk = smem_u32(stages + stage * stage_bytes);
            const uint32_t sv = sk + ktile_bytes;
            const bool partial = rows < T;  // rows past the end hold stale bytes

            // S = K . Qs^T for this warp's m-tiles
            float sc[MTW][NT][4];
#pragma unroll
            for (int mw = 0; mw < MTW; ++mw) {
                const uint32_t mt = (uint32_t)(ph + mw * (int)nph);
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
                    const uint32_t mt = (uint32_t)(ph + mw * (int)nph);
                    sv_[mw][nt][0] = pos_of(mt, g) < rows ? sc[mw][nt][0] + sc[mw][nt][1] : NEG_INF;
                    sv_[mw][nt][1] = pos_of(mt, g + 8) < rows ? sc[mw][nt][2] + sc[mw][nt][3] : NEG_INF;
                    mx = fmax3(mx, sv_[mw][nt][0], sv_[mw][nt][1]);
                }
                mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 16));
                float mn = m_run[nt];
                if (m_run[nt] == NEG_INF || mx > m_run[nt] + kRescaleThreshold) mn = fmaxf(m_run[nt], mx);
                m_use[nt] = mn == NEG_INF ? 0.f : mn;
                alpha[nt] = m_run[nt] == NEG_INF ? 0.f : fast_exp2(m_run[nt] - m_use[nt]);
                moved |= !fresh && mn != m_run[nt];
                m_run[nt] = mn;
            }
            if (__any_sync(kFull, moved)) {
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
                const uint32_t mt = (uint32_t)(ph + mw * (int)nph);
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
        }

        // --------------------------------------------------------- merge
        // Items in completion order: the first one claimed by the producer
        // and passed with the end record, each further one by thread 0 after
        // the current one.  Item piece k = item % ips of a sequence is row
        // block k / DS (R rows) and head-dim slice k % DS (D / DS dims).
        const uint32_t rw = R * wpr / NW;  // rows per warp: 1 or 2
        if (threadIdx.x == 0) {
            flags[1] = flags[0] ? kNoItem : end_item;
            flags[2] = end_np;
            flags[4] = end_seq;
        }
        named_bar_sync(1, NW * 32);
        while (true) {
            const uint32_t item = flags[1], np = flags[2], sq = flags[4];
            named_bar_sync(1, NW * 32);  // read before thread 0 writes the next
            if (item >= items) break;
            const uint32_t k = item % ips;
            const uint32_t row0 = k / DS * R, dim0 = k % DS * (D / DS);
            const uint32_t nsub = np * nph;
            if (rw == 2)
                merge_item<D, D / 32, 2, NW>(p, sq, row0, 0u, nsub, nph, 1u, warp, lane, mscr, stages);
            else if (DS == 1)
                merge_item<D, D / 32, 1, NW>(p, sq, row0, 0u, nsub, nph, wpr, warp, lane, mscr, stages);
            else if (DS == 2)
                merge_item<D, D / 64, 1, NW>(p, sq, row0, dim0, nsub, nph, wpr, warp, lane, mscr, stages);
            else if constexpr (D >= 128)
                merge_item<D, D / 128, 1, NW>(p, sq, row0, dim0, nsub, nph, wpr, warp, lane, mscr, stages);
            if (threadIdx.x == 0) {
                uint32_t nxt = kNoItem, nseq = 0, nnp = 0;
                if (!claim_item(p, state, queue, ips, items, flags, nxt, nseq, nnp)) nxt = kNoItem;
                flags[1] = nxt;
                flags[2] = nnp;
                flags[4] = nseq;
            }
            named_bar_sync(1, NW * 32);  // the next item is published; the merge scratch is free
        }
    }

    // The last CTA to leave returns the schedule counters to zero for the
    // next call.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        flags[3] = atomicAdd(&p.sched[0], 1u) == gridDim.x - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (flags[3]) {
        __threadfence();
        // claim counters [0, 256), state words (two u32 each) after them,
        // the completion queue [768, 1024), ended visits [1024, 1280)
        for (uint32_t i = threadIdx.x; i < 5u * kMaxSeqsPerLaunch; i += blockDim.x) {
            const uint32_t sq = i < (uint32_t)kMaxSeqsPerLaunch        ? i
                                : i < 3u * (uint32_t)kMaxSeqsPerLaunch ? (i - kMaxSeqsPerLaunch) / 2u
                                                                       : i % kMaxSeqsPerLaunch;
            if (sq < p.n_seqs) p.counters[i] = 0u;
        }
        for (uint32_t i = threadIdx.x; i < p.n_seqs * p.parts_per_seq; i += blockDim.x) p.part_tiles[i] = 0u;
        __syncthreads();
        if (threadIdx.x == 0) {
            p.sched[1] = 0u;
            p.sched[2] = 0u;
            p.sched[0] = 0u;
            if (p.x_world > 1) *p.x_epoch = exchange_next_epoch(__ldcg(p.x_epoch));  // this call's epoch
            __threadfence();
        }
    }
}

// ----------------------------------------------------------------- host
template <int D, int G, bool F16>
cudaError_t launch_t(const DecodeParams &p, int grid, cudaStream_t stream) {
    constexpr int NW = decode_bulk_warps(D);
    const uint32_t smem = smem_bytes<D, G, NW>(p.rows_per_tile, p.row_bytes);
    if (smem > (uint32_t)kSmemBudget) return cudaErrorNotSupported;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_bulk_kernel<D, G, F16, NW>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    decode_bulk_kernel<D, G, F16, NW><<<grid, BCfg<D, G, NW>::THREADS, smem, stream>>>(p);
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

uint32_t decode_assign_homes(DecodeParams &p, uint32_t grid) {
    const uint32_t n = p.n_seqs;
    uint32_t nt[kMaxSeqsPerLaunch], h[kMaxSeqsPerLaunch], order[kMaxSeqsPerLaunch];
    for (uint32_t s = 0; s < n; ++s) {
        nt[s] = (p.seqs[s].len + p.rows_per_tile - 1) / p.rows_per_tile;
        h[s] = 0;
        order[s] = s;
    }
    std::sort(order, order + n, [&](uint32_t a, uint32_t b) { return nt[a] != nt[b] ? nt[a] > nt[b] : a < b; });
    uint32_t left = grid;
    for (uint32_t i = 0; i < n && left; ++i, --left) h[order[i]] = 1;
    // further CTAs, one at a time, to the most tiles per home (nt / h,
    // compared as nt_a * h_b > nt_b * h_a; lowest index on ties)
    while (left) {
        uint32_t best = n;
        for (uint32_t s = 0; s < n; ++s) {
            if (h[s] == 0 || h[s] >= nt[s]) continue;
            if (best == n || (uint64_t)nt[s] * h[best] > (uint64_t)nt[best] * h[s]) best = s;
        }
        if (best == n) break;  // every sequence has a home per tile
        ++h[best];
        --left;
    }
    uint32_t lo = 0, most = 0;
    for (uint32_t s = 0; s < n; ++s) {
        p.seqs[s].slot_base = lo;
        p.seqs[s].n_slots = h[s];
        lo += h[s];
        most = std::max(most, h[s]);
    }
    return most;
}

bool decode_bulk_supported(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group) {
    if (dt != BML_BF16 && dt != BML_F16) return false;
    if (head_dim != 64 && head_dim != 128) return false;
    if (group != 1 && group != 2 && group != 4 && group != 8) return false;
    if (n_kv != 1 && n_kv != 2 && n_kv != 4 && n_kv != 8) return false;
    // whole m-tiles: T = 32 KiB / row_bytes must be a multiple of 16 and
    // split evenly over the warps of a kv head
    const uint32_t row_bytes = n_kv * head_dim * 2;
    if (row_bytes < 512 || row_bytes > 2048) return false;
    const uint32_t T = kStageK / row_bytes;
    const uint32_t nw = decode_bulk_warps(head_dim);
    if (T % 16 != 0 || nw % n_kv != 0 || (T / 16) % (nw / n_kv) != 0) return false;
    const uint32_t smem = head_dim == 128 ? smem_bytes<128, 8, decode_bulk_warps(128)>(T, row_bytes)
                                          : smem_bytes<64, 8, decode_bulk_warps(64)>(T, row_bytes);
    return smem <= (uint32_t)kSmemBudget;
}

cudaError_t launch_decode_bulk(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group, int grid,
                               cudaStream_t stream) {
    if (!decode_bulk_supported(dt, head_dim, p.n_kv, group)) return cudaErrorNotSupported;
    if (p.rows_per_tile * p.row_bytes != (uint32_t)kStageK || p.row_bytes % 128 != 0 || p.rows_per_tile % 16 != 0)
        return cudaErrorInvalidValue;
    // every CTA starts on a tile; parts, merge items and counters in range
    if (!p.sched || !p.part_tiles || !p.counters || grid <= 0 || (uint32_t)grid > p.total_tiles ||
        p.n_seqs == 0 || p.n_seqs > (uint32_t)kMaxSeqsPerLaunch || p.parts_per_seq == 0 ||
        (size_t)p.n_seqs * p.parts_per_seq > kMaxPartTiles || p.claim_tiles == 0)
        return cudaErrorInvalidValue;
    // merge items: wpr warps per row and 1 or 2 rows per warp (2 only with
    // one warp per row), whole items per sequence
    const uint32_t wpr = p.merge_wpr, R = p.merge_rows;
    const uint32_t DS = p.merge_dsplit;
    const uint32_t NW = decode_bulk_warps(head_dim);
    if (!(wpr == 1 || wpr == 2 || wpr == 4 || wpr == 8 || wpr == 16) || wpr > NW ||
        !(R * wpr == NW || (wpr == 1 && R == 2u * NW)) ||
        p.n_heads % R != 0 || !(DS == 1 || DS == 2 || DS == 4) || 32u * DS > head_dim ||
        (DS > 1 && R * wpr != NW))
        return cudaErrorInvalidValue;
    // a KV split over GPUs: one sequence, items of one row x 32 dims
    if (p.x_world > 1 && (p.x_world > (uint32_t)kMaxExchangeRanks || p.x_rank >= p.x_world || p.n_seqs != 1 ||
                          p.mode != kModeFinal || DS * 32u != head_dim || wpr != NW || R != 1 ||
                          p.x_units != p.n_heads * DS || p.x_epoch == nullptr))
        return cudaErrorInvalidValue;
    // the home CTAs: contiguous ranges covering the grid, each home CTA's
    // static tile and part inside its sequence
    uint32_t lo = 0;
    for (uint32_t s = 0; s < p.n_seqs; ++s) {
        const DecodeSeq &q = p.seqs[s];
        if (q.slot_base != lo || q.n_slots > p.parts_per_seq || q.n_slots > (q.len + p.rows_per_tile - 1) / p.rows_per_tile)
            return cudaErrorInvalidValue;
        lo += q.n_slots;
    }
    if (lo != (uint32_t)grid) return cudaErrorInvalidValue;
    const bool f16 = dt == BML_F16;
    if (head_dim == 128) return f16 ? launch_g<128, true>(p, group, grid, stream) : launch_g<128, false>(p, group, grid, stream);
    return f16 ? launch_g<64, true>(p, group, grid, stream) : launch_g<64, false>(p, group, grid, stream);
}

}  // namespace bml
