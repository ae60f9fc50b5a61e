// Batched decode (B independent sequences sharing one weight image):
// argument structs of the tcgen05 W4A8 GEMM and its per-sequence prologue /
// epilogue kernels, and of the batched vector kernels.  See f5_bgemm.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "f5_kernels.cuh"

namespace f5 {

constexpr int BG_MAX_SEG = 4;
constexpr int BG_TILE = 128;     // weight rows per MMA tile (tcgen05 M)
constexpr int BG_GPS = 4;        // groups of 128 k per pipeline stage

// One weight image of a batched GEMM op.  Tiles never straddle segments.
struct BgemmSeg {
  const uint8_t *w;   // packed rows (ref/w4a8_ref.py:102-114 wire format)
  int rows;
  int tile_begin;     // first tile of this segment in the op's tile list
  int p_row0;         // first row of this segment in the p scratch
  int argmax;         // LM head: per-sequence running argmax of y32 (no p rows)
};

// 128-byte opaque CUtensorMap (cuTensorMapEncodeTiled): the packed image as
// a 2D uint8 tensor {row bytes, rows}, box {256 bytes, 128 rows}, zero fill
struct alignas(64) TmapBytes {
  unsigned char b[128];
};

struct BgemmArgs {
  TmapBytes tmap[BG_MAX_SEG];   // first: kernel-parameter tensor maps must be 64-byte aligned
  BgemmSeg seg[BG_MAX_SEG];
  int nseg, ntiles;
  int K, NG, stride, sh;
  int S;              // K splits: unit = (tile, split), NG / S groups each (multiple of 8)
  int B, Bp;          // sequences, padded MMA N (16, 32 or 64)
  int ns;             // pipeline stages (set by the launcher)
  const int8_t *xt;   // [NG][Bp][128] x8 in the MMA operand layout (see k_bprep)
  int64_t *p;         // [S][Bp][ptot] partial p = sum_g m_g * acc_g over the split's groups
  int ptot;
  unsigned long long *key;   // [Bp] argmax keys (argmax segments)
  uint32_t *err;
  int32_t *y_out;     // argmax segments, optional: y32 of every row, y_out[b * y_bs + row]
  long long y_bs;
  unsigned long long *trace; // optional globaltimer marks of CTA 0, 10240 words: [0,1024) stage
                             // issued, [1024,2048) stage unpack start, then per group [2048,4096)
                             // unpacked, [4096,6144) MMA issued, [6144,8192) accumulator ready,
                             // [8192,10240) accumulator folded
};

// Per-sequence prologue: the decode path's fused GEMV prologue (RMSNorm /
// DYNQ8 / gated attention) for sequence blockIdx.y, written as the GEMM's
// B operand.  pro.src / src2 / dbg point at sequence 0; *_bs are byte
// strides between sequences.
struct BprepArgs {
  GemvPrologue pro;
  long long src_bs, src2_bs;
  int K, NG, B, Bp;
  const int8_t *x8_in;   // PRO_X8: [B][K] quantized inputs (xmeta_in nullable)
  const int *xmeta_in;
  int8_t *x8;            // [Bp][K] natural-order copy (API / debug)
  int *xmeta;            // [Bp][2] {e_x, in_f}
  int8_t *xt;
  uint32_t *err;
};

// Per-sequence epilogue of a batched GEMM op: sums the S partials of p and
// applies the GEMV epilogue of the segment's mode (GM_*) for every
// (sequence, row).  g.seg[] holds the sequence-0 pointers; out_bs / aux_bs /
// ring_bs are byte strides between sequences.
struct BepiSeg {
  int p_row0, p_row0_up;   // p rows of the segment (and of the paired up rows)
  long long out_bs, aux_bs, ring_bs, pout_bs;
};
struct BepiArgs {
  GemvArgs g;              // seg[i].unit_begin = first unit (row, or row pair) of segment i
  BepiSeg bs[GEMV_MAX_SEG];
  int S, B, Bp, ptot;
  const int64_t *p;
  const int *xmeta;        // [Bp][2]
  StepParams *params;      // [B] (GM_CONV reads params[b].T)
};

// tensor map of a packed image (rows of `stride` bytes) for the GEMM's
// weight stages; false if the driver refuses it
bool bgemm_tmap(TmapBytes *out, const uint8_t *w, int rows, int stride);
unsigned long long *&bgemm_trace_buffer();
constexpr int BG_TRACE_WORDS = 10240;
cudaError_t launch_bprep(const BprepArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_bgemm(BgemmArgs a, cudaStream_t st, bool pdl, int max_ctas);
cudaError_t launch_bepi(const BepiArgs &a, cudaStream_t st, bool pdl);
// K splits for a GEMM of `tiles` tiles and NG groups on `ctas` CTAs
int bgemm_splits(int tiles, int NG, int ctas, bool argmax);
size_t bgemm_smem(int Bp, int *ns);

}  // namespace f5
