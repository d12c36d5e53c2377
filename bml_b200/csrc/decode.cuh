// decode.cuh -- launch interface of the split-K flash-decoding kernels.
#pragma once

#include "common.cuh"

namespace bml {

// Per-sequence entry of a decode launch (host-computed schedule).
// Static schedule (decode_kernel): CTA b owns global tiles
// [b*tiles_per_cta, (b+1)*tiles_per_cta); tile_begin is the sequence's first
// global tile and its n_slots partial slots are one per CTA touching it.
// Claimed schedule (decode_bulk_kernel): tile_begin is the sequence's first
// global tile (prefix of the tile counts); slot_base / n_slots are the first
// of its home CTAs and their number (decode_assign_homes); CTAs claim the
// sequence's tiles at run time and leave at most parts_per_seq parts of it.
struct DecodeSeq {
    const void *k;        // [len][n_kv][D]
    const void *v;
    uint32_t len;         // positions attended
    uint32_t tile_begin;  // first global tile of this sequence
    uint32_t slot_base;   // static: first partial slot; claimed: first home CTA
    uint32_t n_slots;     // static: CTAs touching it; claimed: home CTAs
};

constexpr int kMaxSeqsPerLaunch = 256;

// KV split over GPUs: at most 8 ranks; a unit is (M, L, 2 spare, 32 dims)
constexpr int kMaxExchangeRanks = 8;
constexpr int kExchangeUnitFloats = 36;
// Exchange buffer of a rank: data [2 call parities][kMaxExchangeRanks][units]
// units of kExchangeUnitFloats, then flags [2][kMaxExchangeRanks][units] u32,
// then the rank's call counter (u32; the epoch of its last call, 0 before
// the first), kept on the device so that a launch captured in a CUDA graph
// takes a new epoch at every replay.
__host__ __device__ inline size_t exchange_data_floats(uint32_t units) {
    return 2ull * kMaxExchangeRanks * units * kExchangeUnitFloats;
}
inline size_t exchange_epoch_offset(uint32_t units) {
    return exchange_data_floats(units) * 4 + 2ull * kMaxExchangeRanks * units * 4;
}
inline size_t exchange_bytes(uint32_t units) { return exchange_epoch_offset(units) + 16; }
// The epoch a call takes after `last`: never 0 (flags start at 0).
__host__ __device__ inline uint32_t exchange_next_epoch(uint32_t last) { return last + 1u == 0u ? 1u : last + 1u; }

enum DecodeMode : int { kModeFinal = 0, kModePartial = 1 };

// Test-only behaviour of decode_bulk_kernel (bml_diag_decode_batched): the
// producer arms no stage, so every consumer wait runs into its limit.
constexpr uint32_t kDiagStall = 1u;

struct DecodeParams {
    const float *q;        // [n_seqs][n_heads][D] f32
    float *out;            // final outputs [n_seqs][n_heads][D]
    float *part_m;         // partial-mode outputs [n_seqs][n_heads]
    float *part_l;
    float *part_o;         // [n_seqs][n_heads][D]
    float *slot_ml;        // scratch [n_slots][n_heads][2]
    float *slot_o;         // scratch [n_slots][n_heads][D]
    uint32_t *counters;    // scratch [5][kMaxSeqsPerLaunch] words, zero between calls
    uint32_t *err;         // scratch error word
    uint32_t n_seqs, n_heads, n_kv;
    uint32_t rows_per_tile;   // T
    uint32_t total_tiles;
    uint32_t tiles_per_cta;   // static schedule
    uint32_t row_bytes;       // n_kv * D * sizeof(elem)
    float qscale;             // scale * log2(e)
    int mode;
    int merge_in_kernel;      // static schedule: 1 = the last CTA of a sequence
                              // merges its slots, 0 = launch_slot_merge does
    // claimed schedule (decode_bulk_kernel)
    uint32_t *sched;          // [0] CTA exit ticket, [1] merge items claimed, [2] sequences
                              // completed; zero between calls
    uint32_t *part_tiles;     // [n_seqs * parts_per_seq] tiles in each part (0: empty); zero between calls
    uint32_t parts_per_seq;   // parts a sequence may have (>= 1)
    uint32_t claim_tiles;     // tiles per claim
    uint32_t join_min;        // unclaimed tiles per CTA on a started sequence that make it worth joining
    uint32_t merge_rows;      // q-head rows per merge item (1, 2, 4, 8 or 16)
    uint32_t merge_wpr;       // consumer warps sharing one row in the merge (1, 2, 4 or 8)
    uint32_t merge_dsplit;    // head-dim slices of a row block, one merge item each (1, 2 or 4)
    uint32_t diag;            // kDiag* flags, 0 outside tests
    uint64_t wait_ns;         // limit of every bounded wait
    // KV split over GPUs (x_world > 1; one sequence a launch): each merge
    // item is one exchange unit (q-head row, 32 head dims); its rank's (M, L,
    // O / L) goes to every rank's exchange buffer over peer memory, and the
    // output is merged from all ranks' units in rank order.  x_epoch: this
    // rank's call counter in its own exchange buffer; the launch's epoch is
    // the next value, and the launch's last CTA stores it back.
    uint32_t x_world, x_rank, x_units;
    uint32_t *x_epoch;
    float *x_base[kMaxExchangeRanks];  // every rank's exchange buffer, mapped here
    DecodeSeq seqs[kMaxSeqsPerLaunch];
};

// Scratch layout inside a caller workspace.
struct DecodeWorkspace {
    uint32_t *err;
    uint32_t *sched;
    uint32_t *counters;
    uint32_t *part_tiles;
    float *slot_ml;
    float *slot_o;
    size_t max_slots;
};

// Recommended scratch bytes and the minimum a call accepts.  A slot holds
// one partial (m, l, o) for every q head of a sequence.
size_t decode_workspace_bytes(uint32_t n_seqs, uint32_t n_heads, uint32_t head_dim,
                              int num_sms);
size_t decode_workspace_min_bytes(uint32_t n_seqs, uint32_t n_heads, uint32_t n_kv, uint32_t head_dim,
                                  int num_sms);
// Bytes at the start of a workspace that must be zero before a call (error
// word, schedule counters, part tile counts); every call leaves all but the
// error word zero, and the error word keeps a timeout until it is checked.
size_t decode_workspace_zero_bytes();
bool decode_workspace_carve(void *ws, size_t bytes, uint32_t n_seqs, uint32_t n_heads, uint32_t n_kv,
                            uint32_t head_dim, int num_sms, DecodeWorkspace *out);

// Rows of one tile for a (dtype, head_dim, n_kv) combination.
uint32_t decode_rows_per_tile(bml_dtype dt, uint32_t head_dim, uint32_t n_kv);

enum DecodeKernel : int { kKernBulk = 1, kKernCuda = 3 };

// The kernel a launch takes for a shape: the bulk-copy warp-MMA kernel
// (claimed schedule, in-kernel merge) for 16-bit caches with 512..2048-byte
// position rows, the CUDA-core kernel (static schedule) for the rest.
DecodeKernel decode_select(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group);

// Launches the CUDA-core kernel; returns a CUDA error code.
cudaError_t launch_decode(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group, int grid,
                          cudaStream_t stream);

// Group bulk copies into staggered shared-memory rows, warp-level MMAs, tiles
// claimed at run time and partials merged in the same launch
// (decode_bulk.cu); 256 sequences a launch.
bool decode_bulk_supported(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group);
cudaError_t launch_decode_bulk(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group,
                               int grid, cudaStream_t stream);
// Claimed schedule: deals the grid's CTAs to the sequences of p as home
// CTAs (contiguous ranges in sequence order, seqs[].slot_base / n_slots) so
// that the largest home load, tiles per home CTA, is as small as it can be:
// one home for each sequence (longest first, while CTAs last), then each
// further CTA to the sequence with the most tiles per home; never more homes
// than tiles.  Home CTAs take a sequence's first tiles and parts statically,
// one each, so a launch issues its first copies without waiting on an
// atomic.  Returns the most homes any sequence got.  Measured on B200: the
// even spacing it replaces (CTA b's home held tile (b + 1/2) * total / grid)
// gave a 27-tile sequence of the ragged TinyLlama-shaped batch one home CTA
// against an average of 15.3 tiles, and that CTA set the batch's time.
uint32_t decode_assign_homes(DecodeParams &p, uint32_t grid);

// Parts of a claimed-schedule launch (n_seqs * parts_per_seq) are limited
// by the fixed part-tile area of a workspace.
constexpr size_t kMaxPartTiles = 16384;
// Consumer warps of decode_bulk_kernel: 16 for head_dim 64 (tiles of 64
// positions carry twice the MMA work per byte of head_dim 128, and a warp's
// dependent chain per tile is what limits them: measured on B200, 8 warps
// streamed the ragged TinyLlama-shaped batch at ~4.6 TB/s against 7.3 for
// head_dim 128), 8 otherwise (the register budget of 17 warps, 96 a
// thread, does not hold the head_dim-128 state).
__host__ __device__ constexpr uint32_t decode_bulk_warps(uint32_t head_dim) { return head_dim == 64 ? 16u : 8u; }
// Partial slots a q head row of a sequence leaves per part: the consumer
// warps serving one kv head.
inline uint32_t decode_bulk_phases(uint32_t n_kv, uint32_t head_dim) { return decode_bulk_warps(head_dim) / n_kv; }

// Merge of split-K slots for sequences spread over more CTAs than the
// in-kernel merge handles well; one CTA per (sequence, head) row.
cudaError_t launch_slot_merge(const DecodeParams &p, uint32_t head_dim, cudaStream_t stream);

// A sequence spanning more CTAs than this has its slots merged by
// launch_slot_merge instead of by its last CTA.
constexpr uint32_t kInKernelMergeMaxSlots = 8;

// merge_lse with each part's weight multiplied by counts[i] (at most 2
// parts): the ring-wrap decode's slots visited c+1 and c times.
cudaError_t launch_merge_counted(const float *m, const float *l, const float *o, uint32_t n_parts,
                                 const float *counts, uint32_t n_rows, uint32_t head_dim, float *out,
                                 cudaStream_t stream);

cudaError_t launch_merge_lse(const float *m, const float *l, const float *o, uint32_t n_parts,
                             uint32_t n_rows, uint32_t head_dim, float *out,
                             cudaStream_t stream);

cudaError_t launch_merge_lse_packed(const float *parts, uint32_t n_parts, uint32_t n_rows,
                                    uint32_t head_dim, float *out, cudaStream_t stream);

}  // namespace bml
