// decode.cuh -- launch interface of the split-K flash-decoding kernels.
#pragma once

#include "common.cuh"

namespace bml {

// Per-sequence entry of a decode launch (host-computed schedule).
// Static schedule (chunk_tiles == 0): CTA b owns global tiles
// [b*tiles_per_cta, (b+1)*tiles_per_cta); tile_begin is the sequence's first
// global tile and its n_slots partial slots are one per CTA touching it.
// Dynamic schedule (chunk_tiles > 0): the sequence is cut into n_slots
// chunks of chunk_tiles tiles, global chunk indices [tile_begin, tile_begin
// + n_slots); CTAs claim chunks at run time and chunk c leaves its partial
// in slot c (slot_base == tile_begin).
struct DecodeSeq {
    const void *k;        // [len][n_kv][D]
    const void *v;
    uint32_t len;         // positions attended
    uint32_t tile_begin;  // first global tile (static) or chunk (dynamic)
    uint32_t slot_base;   // first partial slot of this sequence
    uint32_t n_slots;     // CTAs (static) or chunks (dynamic) of this sequence
};

constexpr int kMaxSeqsPerLaunch = 256;

enum DecodeMode : int { kModeFinal = 0, kModePartial = 1 };

struct DecodeParams {
    const float *q;        // [n_seqs][n_heads][D] f32
    float *out;            // final outputs [n_seqs][n_heads][D]
    float *part_m;         // partial-mode outputs [n_seqs][n_heads]
    float *part_l;
    float *part_o;         // [n_seqs][n_heads][D]
    float *slot_ml;        // scratch [n_slots][n_heads][2]
    float *slot_o;         // scratch [n_slots][n_heads][D]
    uint32_t *counters;    // scratch [n_seqs], zero between calls
    uint32_t *err;         // scratch error word
    uint32_t n_seqs, n_heads, n_kv;
    uint32_t rows_per_tile;   // T
    uint32_t total_tiles;
    uint32_t tiles_per_cta;
    uint32_t row_bytes;       // n_kv * D * sizeof(elem)
    float qscale;             // scale * log2(e)
    int mode;
    int merge_in_kernel;      // 1: last CTA of a sequence merges its slots;
                              // 0: slots are merged by launch_slot_merge
    uint32_t chunk_tiles;     // dynamic schedule: tiles per chunk (0: static)
    uint32_t total_chunks;
    uint32_t *sched;          // dynamic schedule: [0] chunk claims, [1] CTA exit
                              // ticket; zero between calls
    DecodeSeq seqs[kMaxSeqsPerLaunch];
};

// Scratch layout inside a caller workspace.
struct DecodeWorkspace {
    uint32_t *err;
    uint32_t *sched;
    uint32_t *counters;
    float *slot_ml;
    float *slot_o;
    size_t max_slots;
};

// Recommended scratch bytes (room for the dynamic schedule's chunk slots)
// and the minimum a call accepts (the static schedule's slots); the
// dynamic schedule sizes its chunks to the slots a workspace holds.
size_t decode_workspace_bytes(uint32_t n_seqs, uint32_t n_heads, uint32_t head_dim,
                              int num_sms);
size_t decode_workspace_min_bytes(uint32_t n_seqs, uint32_t n_heads, uint32_t head_dim,
                                  int num_sms);
// Bytes at the start of a workspace that must be zero before a call
// (error word and merge tickets).
size_t decode_workspace_zero_bytes();
bool decode_workspace_carve(void *ws, size_t bytes, uint32_t n_seqs, uint32_t n_heads,
                            uint32_t head_dim, int num_sms, DecodeWorkspace *out);

// Rows of one tile for a (dtype, head_dim, n_kv) combination.
uint32_t decode_rows_per_tile(bml_dtype dt, uint32_t head_dim, uint32_t n_kv);

enum DecodeKernel : int { kKernTma = 0, kKernBulk = 1, kKernMma = 2, kKernCuda = 3 };

// The kernel a launch takes, from the shape, the family override and the
// sequences of p (n_seqs, n_kv and seqs[].k / v / len filled in).  The
// bulk-copy kernel runs the dynamic schedule, every other kernel the static
// one.
DecodeKernel decode_select(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group);

// Launches the selected decode kernel; returns a CUDA error code.
cudaError_t launch_decode(const DecodeParams &p, DecodeKernel kern, bml_dtype dt, uint32_t head_dim,
                          uint32_t group, int grid, cudaStream_t stream);

// Tensor-core (mma.sync m16n8k16) variant for 16-bit caches, same
// parameters and schedule (decode_mma.cu).  launch_decode dispatches to it
// for the shapes decode_mma_supported accepts.
bool decode_mma_supported(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group);
cudaError_t launch_decode_mma(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group,
                              int grid, cudaStream_t stream);

// Same arithmetic with K/V brought in by TMA through per-sequence tensor
// maps (decode_tma.cu); at most decode_tma_max_seqs() sequences a launch.
// launch_decode prefers it where supported; cudaErrorNotSupported means the
// caller should fall back.
bool decode_tma_supported(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group);
uint32_t decode_tma_max_seqs();

// Same arithmetic with tiles brought in by group bulk copies into staggered
// shared-memory rows and chunks of tiles claimed at run time (decode_bulk.cu,
// dynamic schedule only); 256 sequences a launch.
bool decode_bulk_supported(bml_dtype dt, uint32_t head_dim, uint32_t n_kv, uint32_t group);
cudaError_t launch_decode_bulk(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group,
                               int grid, cudaStream_t stream);

// Kernel family for 16-bit caches.  By default (kDecodeAuto) the bulk-copy
// kernel with the dynamic schedule; BML_DECODE_KERNEL=tma,
// =bulk, =mma or =cuda in the environment (read once) forces the TMA, bulk-
// copy, cp.async warp-MMA or CUDA-core kernel -- for tests and comparisons.
enum DecodeFamily : int { kDecodeAuto = 0, kDecodeMma = 1, kDecodeCuda = 2, kDecodeBulk = 3, kDecodeTma = 4 };
DecodeFamily decode_family_override();
cudaError_t launch_decode_tma(const DecodeParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group,
                              int grid, cudaStream_t stream);

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
