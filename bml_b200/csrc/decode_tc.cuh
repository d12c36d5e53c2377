// decode_tc.cuh -- launch interface of the tcgen05 decode kernel.
#pragma once

#include "decode.cuh"

namespace bml {

struct TcSeq {
    const void *k;            // [len][n_kv][D] 16-bit
    const void *v;
    uint32_t len;
    uint32_t tiles;           // ceil(len / 128): tiles of each (sequence, kv head) unit
    uint32_t tile_begin;      // global tile index of unit (this sequence, kv head 0)
    uint32_t slot_base;       // first partial slot of unit (this sequence, kv head 0)
    uint32_t slots_per_unit;  // slot stride between kv heads of this sequence
    uint32_t pad_;
};

struct TcParams {
    const float *q;       // [n_seqs][n_heads][D] f32
    float *out;           // final outputs
    float *part_m, *part_l, *part_o;  // partial-mode outputs
    float *slot_ml;       // scratch [slots][G][2]
    float *slot_o;        // scratch [slots][G][D]
    uint32_t *counters;   // scratch [n_seqs * n_kv], zero between calls
    uint32_t *err;
    uint32_t n_seqs, n_heads, n_kv;
    uint32_t total_tiles, tiles_per_cta;
    uint32_t row_bytes;   // n_kv * D * 2
    float qscale;         // scale * log2(e)
    int mode;
    TcSeq seqs[kMaxSeqsPerLaunch];
};

bool decode_tc_supported(bml_dtype dt, uint32_t head_dim, uint32_t group);

cudaError_t launch_decode_tc(const TcParams &p, bml_dtype dt, uint32_t head_dim, uint32_t group, int grid,
                             cudaStream_t stream);

}  // namespace bml
