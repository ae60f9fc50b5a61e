// Batched W4A8 decode GEMM on the 5th-generation tensor cores (sm_100a).
//
// B independent sequences share one weight image, so every projection of
// the decode step becomes Y[b][row] = matvec_y32(w4, m, sh, x8[b])
// (ref/w4a8_ref.py:254-289) for b < B:
//   acc_g[row][b] = sum_{k in g} w4[row][k] * x8[b][k]       (int32, |.| <= 2^17)
//   p[row][b]     = sum_g m_g[row] * acc_g[row][b]            (int64)
//   y32           = rshift_round(p, sh)
// acc_g is a 128 x Bp x 128 int8 matrix product per group: tcgen05.mma
// kind::i8 with an int32 accumulator in tensor memory (TMEM), one MMA tile
// of 128 weight rows x Bp sequences per group.  The group scale is applied
// by the epilogue warps, which read each group's accumulator out of TMEM and
// fold m_g * acc_g into int64 registers (a different m_g per row and group
// rules out accumulating across groups inside the MMA).
//
// The weights stay in the reference's packed row format in HBM.  A stage
// brings 4 groups (256 bytes) of each of the tile's 128 rows into shared
// memory as two 2D tensor-map boxes (128 rows x 128 bytes, 128-byte
// swizzle).  Four unpack warps, one per tensor-memory lane quarter, turn a
// row's nibbles into 16 * w4 as signed bytes ((word << 4) & 0xF0F0F0F0 for
// even k, word & 0xF0F0F0F0 for odd k) and store them straight into tensor
// memory with tcgen05.st: the MMA reads its A operand (128 rows x 32 bytes
// of K per instruction) from tensor memory, so the unpacked weights never
// touch shared memory.  The accumulator holds 16 * acc_g (|.| <= 2^21) and
// p = (sum_g m_g * 16 acc_g) >> 4 exactly.  Within each 8-weight block the
// unpacked bytes are the even k then the odd k; the prologue writes x8 (the
// B operand, 128-byte-swizzled K-major rows in shared memory) in the same
// order.
//
// Warp roles (one CTA per SM): warp 0 streams the stages,
// warp 1 allocates tensor memory and issues the MMAs (one thread: 4
// tcgen05.mma kind::i8 M=128 N=Bp K=32 per group, A from one of 2-4 A
// buffers into one of up to 4 accumulator buffers, tcgen05.commit to
// mbarriers), warps 2-5 unpack, Bp / 4
// fold warps from warp 6 read each group's accumulator back (lane quarter =
// warp % 4, 16-column block = (warp - 6) / 4) and fold m_g * acc_g into
// int64 registers.
// Every hand-off is an mbarrier; every wait is bounded and an expired wait
// sets DERR_TIMEOUT and unwinds the CTA (no copy or MMA left in flight).
//
// Work: units = (128-row tile, K split); split s covers groups
// [s*NG/S, (s+1)*NG/S) and writes its partial p to p[s][b][row]; k_bepi
// sums the S partials (integer addition: exact in any order) and runs the
// per-sequence epilogue of the op.  The LM head (S = 1) reduces its
// argmax inside the GEMM, per CTA in shared memory, then one atomicMax per
// sequence.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "f5_batch.cuh"
#include "f5_block.cuh"
#include "f5_bprep.cuh"
#include "f5_gemv_core.cuh"
#include "f5_tc.cuh"

namespace f5 {

constexpr int BG_MMAW = 1;         // MMA warp 1 (one issuing thread)
constexpr int BG_UNPACK = 4;       // unpack warps 2-5 (one per TMEM lane quarter)
constexpr int BG_U0 = 1 + BG_MMAW, BG_F0 = BG_U0 + BG_UNPACK;   // first unpack / fold warp
constexpr int BG_FOLDQ = 16;       // accumulator columns per fold thread: Bp / 16 fold warps per lane quarter
constexpr int bg_fold_warps(int Bp) { return 4 * (Bp / BG_FOLDQ); }
constexpr int bg_threads(int Bp) { return 32 * (BG_F0 + bg_fold_warps(Bp)); }
constexpr int BG_MAX_NS = 6;       // pipeline stages at most
constexpr int BG_WBYTES = BG_TILE * 64 * BG_GPS;   // packed weights per stage (32 KB: two 16 KB boxes)
constexpr int BG_SMEM_MAX = 232448 - 4096;
constexpr unsigned long long BG_WAIT_NS = 2000000000ull;

F5_DEV int bg_seg_of_tile(const BgemmArgs &a, int tile) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < BG_MAX_SEG; ++i)
    if (i < a.nseg && tile >= a.seg[i].tile_begin) s = i;
  return s;
}

template <int BP>
__global__ void __launch_bounds__(bg_threads(BP), 1) k_bgemm(const __grid_constant__ BgemmArgs a) {
  constexpr int BPQ = BG_FOLDQ;                             // accumulator columns per fold thread
  constexpr int BG_FOLD = bg_fold_warps(BP);
  constexpr int XBYTES = BP * 128 * BG_GPS;
  constexpr int STAGE = BG_WBYTES + XBYTES;
  // tensor memory: NA A buffers of a group pair (64 columns each) at column
  // 0, then ND accumulator buffers of a pair (2 x BP columns each).  A and
  // accumulator buffers recycle independently: the unpack reuses an A buffer
  // once the MMAs that read it completed, the MMA reuses an accumulator
  // buffer once the fold read it back.
  constexpr int NA = BP <= 16 ? 4 : (BP <= 32 ? 3 : 2);
  constexpr int DCOL = 2 * BP;
  constexpr int ND = (512 - 64 * NA) / DCOL > 4 ? 4 : (512 - 64 * NA) / DCOL;
  // NA == ND (Bp = 16): the unpack waits until the fold read back pair
  // pc - NA, which frees both its A and its accumulators, and the MMA thread
  // (the bottleneck at small N) waits only for A.  NA < ND: the unpack waits
  // for the MMAs of pc - NA, the MMA thread for the fold of pc - ND.
  constexpr bool COUPLED = NA == ND;
  static_assert(ND >= 2 && NA <= ND, "two accumulator buffers at least, no more A buffers than accumulators");
  extern __shared__ uint8_t bg_dyn[];
  __shared__ __align__(8) uint64_t full[BG_MAX_NS], empty[BG_MAX_NS], afull[NA], done[4], tfree[4];
  __shared__ __align__(8) uint64_t drain;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;
  __shared__ unsigned long long s_key[BP];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = a.ns;
  uint8_t *stg = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(bg_dyn) + 1023) & ~(uintptr_t)1023);
  const int gpu = a.NG / a.S;                              // groups per unit
  const int spu = gpu / BG_GPS;                            // stages per unit
  const int ppu = gpu / 2;                                 // group pairs per unit
  const int units = a.ntiles * a.S;
  const bool tr = a.trace && blockIdx.x == 0;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], BG_UNPACK + BG_MMAW);   // every unpack warp + every MMA warp's commit
    }
    for (int i = 0; i < NA; ++i) mbar_init(&afull[i], BG_UNPACK);   // both groups' A written
    for (int i = 0; i < ND; ++i) {
      mbar_init(&done[i], 1);            // both groups' MMAs complete (commit)
      mbar_init(&tfree[i], BG_FOLD);     // both accumulators read back
    }
    mbar_init(&drain, BG_MMAW);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid < BP) s_key[tid] = 0ull;
  if (warp == 1) tc_alloc(&s_tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ---------------- producer: two 128-byte-swizzled weight boxes + the x tiles per stage ----------------
    int sc = 0;
    for (int u = blockIdx.x; u < units && !s_abort; u += gridDim.x) {
      const int tile = u / a.S, sp = u % a.S;
      const int si = bg_seg_of_tile(a, tile);
      const int r0 = (tile - a.seg[si].tile_begin) * BG_TILE;
      for (int st = 0; st < spu; ++st, ++sc) {
        const int s = sc % NS;
        bool ok = true;
        if (lane == 0 && sc >= NS) ok = mbar_wait(&empty[s], ((sc / NS) - 1) & 1, BG_WAIT_NS);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok || s_abort) {
          if (lane == 0 && !ok) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); }
          break;
        }
        const int g = sp * gpu + st * BG_GPS;
        uint8_t *dst = stg + (size_t)s * STAGE;
        if (tr && lane == 0 && sc < 1024) a.trace[sc] = gtimer();
        if (lane == 0) {
          // rows past the image read as zeros
          mbar_expect_tx(&full[s], (uint32_t)STAGE);
          tma_load_2d_stream(dst, &a.tmap[si], g * 64, r0, &full[s]);
          tma_load_2d_stream(dst + BG_WBYTES / 2, &a.tmap[si], g * 64 + 128, r0, &full[s]);
          bulk_g2s(dst + BG_WBYTES, a.xt + (size_t)g * BP * 128, XBYTES, &full[s]);
        }
        __syncwarp();
      }
    }
    if (lane == 0 && s_abort)
      for (int i = max(0, sc - NS); i < sc; ++i) mbar_wait(&full[i % NS], (i / NS) & 1, BG_WAIT_NS);
  } else if (warp == 1) {
    // ---------------- MMA issuer (one thread): one wait, 8 MMAs, one commit per group pair ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_s8s8(BG_TILE, BP);
      int sc = 0, pc = 0;
      for (int u = blockIdx.x; u < units && !s_abort; u += gridDim.x) {
        for (int st = 0; st < spu && !s_abort; ++st, ++sc) {
          const int s = sc % NS;
          if (!mbar_wait(&full[s], (sc / NS) & 1, BG_WAIT_NS)) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); break; }
          const uint64_t bd0 = sw128_desc(smem_u32(stg + (size_t)s * STAGE + BG_WBYTES));
          for (int pi = 0; pi < BG_GPS / 2; ++pi, ++pc) {
            const int ja = pc % NA, jd = pc % ND;
            // afull implies the unpack saw this A buffer's previous MMAs complete
            if (!mbar_wait(&afull[ja], (pc / NA) & 1, BG_WAIT_NS) ||
                (!COUPLED && pc >= ND && !mbar_wait(&tfree[jd], ((pc / ND) - 1) & 1, BG_WAIT_NS))) {
              s_abort = 1;
              atomicOr(a.err, DERR_TIMEOUT);
              break;
            }
            tc_fence_after();
            const uint32_t abase = tmem + (uint32_t)(64 * ja), dbase = tmem + (uint32_t)(64 * NA + jd * DCOL);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const uint64_t bd = bd0 + (uint64_t)(((2 * pi + e) * BP * 128) >> 4);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                tc_mma_i8_ts(dbase + (uint32_t)(e * BP), abase + (uint32_t)(32 * e + 8 * k), bd + 2 * k, idesc,
                             k > 0);
            }
            if (tr && pc < 2048) a.trace[4096 + pc] = gtimer();
            tc_commit(&done[jd]);
          }
          tc_commit(&empty[s]);
        }
      }
      // a commit with no MMA before it arrives at once: the drain completes
      // when every issued MMA has
      tc_commit(&drain);
      mbar_wait(&drain, 0, BG_WAIT_NS);
    }
    __syncwarp();
  } else if (warp < BG_F0) {
    // ---------------- unpack (warps 5-8, one per TMEM lane quarter): thread = row ----------------
    // Row r's packed group gi is 64 bytes = 16-byte chunks 4 (gi & 1) + c of
    // the 128-byte swizzled row r of box gi / 2 (chunk j at j ^ (r & 7)):
    // eight consecutive rows read eight different bank groups.  Nibbles
    // become 16 w as signed bytes ((w << 4) & 0xF0F0F0F0 even k, w &
    // 0xF0F0F0F0 odd k), written to the row's lane of the pair slot's A
    // columns: column 2i = the even k of packed word i, 2i + 1 the odd k.
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
    bool ok = true;
    int sc = 0, pc = 0;
    for (int u = blockIdx.x; u < units && ok && !s_abort; u += gridDim.x) {
      for (int st = 0; st < spu; ++st, ++sc) {
        const int s = sc % NS;
        if (lane == 0) ok = mbar_wait(&full[s], (sc / NS) & 1, BG_WAIT_NS);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (tr && tid == 32 * BG_U0 && sc < 1024) a.trace[1024 + sc] = gtimer();
        if (!ok || s_abort) {
          if (lane == 0 && !ok) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); }
          ok = false;
          break;
        }
        const uint8_t *src = stg + (size_t)s * STAGE + r * 128;
        for (int pi = 0; pi < BG_GPS / 2; ++pi, ++pc) {
          const int j = pc % NA;
          if (pc >= NA) {   // this A buffer's previous pair (pc - NA): its MMAs completed (or, coupled,
            // its accumulators read back); NA <= ND, so the barrier cannot be a phase further on
            if (lane == 0)
              ok = mbar_wait(COUPLED ? &tfree[(pc - NA) % ND] : &done[(pc - NA) % ND], ((pc - NA) / ND) & 1,
                             BG_WAIT_NS);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
              if (lane == 0) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); }
              break;
            }
            tc_fence_after();
          }
          const uint8_t *bx = src + pi * (BG_WBYTES / 2);   // box of groups 2 pi, 2 pi + 1
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            uint32_t o[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int jc = 4 * e + c;
              const uint4 w = *reinterpret_cast<const uint4 *>(bx + ((jc ^ (r & 7)) << 4));
              const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                o[8 * c + 2 * k] = (wv[k] << 4) & 0xF0F0F0F0u;
                o[8 * c + 2 * k + 1] = wv[k] & 0xF0F0F0F0u;
              }
            }
            tc_st32(tq + (uint32_t)(64 * j + 32 * e), o);
          }
          tc_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[j]);
          if (tr && tid == 32 * BG_U0 && pc < 2048) a.trace[2048 + pc] = gtimer();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);   // the stage's packed bytes are consumed
        if (!ok) break;
      }
    }
  } else {
    // ---------------- accumulator fold (warps 6-21) ----------------
    // warp w reads TMEM lane quarter w % 4 (rows 32 (w % 4) + lane) and the
    // 16-column block cq = (w - 6) / 4 of both accumulators of a pair slot
    const int q = warp & 3, cq = (warp - BG_F0) >> 2;
    const int rt = 32 * q + lane;                              // row within the tile
    const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + 64 * NA + (uint32_t)(cq * BPQ);
    int pc = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok && !s_abort; u += gridDim.x) {
      const int tile = u / a.S, sp = u % a.S;
      const BgemmSeg &sg = a.seg[bg_seg_of_tile(a, tile)];
      const int r0 = (tile - sg.tile_begin) * BG_TILE;
      const bool valid = rt < sg.rows - r0;
      long long acc[BPQ];
#pragma unroll
      for (int jj = 0; jj < BPQ; ++jj) acc[jj] = 0;
      // group scales 8 at a time, the next 8 prefetched one block ahead
      const uint4 *ms = reinterpret_cast<const uint4 *>(sg.w + (size_t)(valid ? r0 + rt : r0) * a.stride +
                                                        (size_t)a.NG * 64 + 2 * sp * gpu);
      uint4 mv = __ldg(ms), mvn = gpu > 8 ? __ldg(ms + 1) : make_uint4(0, 0, 0, 0);
      for (int pi = 0; pi < ppu; ++pi, ++pc) {
        const int gi = 2 * pi;
        if ((gi & 7) == 0 && gi) {
          mv = mvn;
          if (gi + 8 < gpu) mvn = __ldg(ms + (gi >> 3) + 1);
        }
        const uint32_t mw = (gi & 6) == 0 ? mv.x : ((gi & 6) == 2 ? mv.y : ((gi & 6) == 4 ? mv.z : mv.w));
        const int32_t m0 = (int32_t)(mw & 0xFFFFu), m1 = (int32_t)(mw >> 16);
        const int j = pc % ND;
        if (lane == 0) ok = mbar_wait(&done[j], (pc / ND) & 1, BG_WAIT_NS);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok || s_abort) {
          if (lane == 0 && !ok) { s_abort = 1; atomicOr(a.err, DERR_TIMEOUT); }
          ok = false;
          break;
        }
        if (tr && warp == BG_F0 && lane == 0 && pc < 2048) a.trace[6144 + pc] = gtimer();
        tc_fence_after();
        int32_t d0[BPQ], d1[BPQ];
        tc_ld<BPQ>(tl + (uint32_t)(j * DCOL), d0);
        tc_ld<BPQ>(tl + (uint32_t)(j * DCOL + BP), d1);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tfree[j]);
#pragma unroll
        for (int jj = 0; jj < BPQ; ++jj) acc[jj] += (long long)m0 * d0[jj] + (long long)m1 * d1[jj];   // 16 p
        if (tr && warp == BG_F0 && lane == 0 && pc < 2048) a.trace[8192 + pc] = gtimer();
      }
      if (!ok) break;
      if (sg.argmax) {
        const int row = r0 + rt;
#pragma unroll
        for (int jj = 0; jj < BPQ; ++jj) {
          const int b = cq * BPQ + jj;
          if (valid && b < a.B) {
            const int32_t y = finish_y32(acc[jj], a.sh, a.err, nullptr);
            atomicMax(&s_key[b], argmax_key(y, row));
            if (a.y_out) a.y_out[(size_t)b * a.y_bs + row] = y;
          }
        }
      } else if (valid) {
        int64_t *po = a.p + ((size_t)sp * BP + cq * BPQ) * a.ptot + sg.p_row0 + r0 + rt;
#pragma unroll
        for (int jj = 0; jj < BPQ; ++jj)
          if (cq * BPQ + jj < a.B) po[(size_t)jj * a.ptot] = acc[jj] >> 4;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tc_dealloc(tmem, 512);
  if (a.key && tid < a.B && s_key[tid]) atomicMax(&a.key[tid], s_key[tid]);
}

// ---------------------------------------------------------------------------
// k_bprep: per-sequence prologue -> the GEMM's B operand
// ---------------------------------------------------------------------------
constexpr int BP_THREADS = 512;

template <int MAXB>
__global__ void __launch_bounds__(BP_THREADS) k_bprep(const __grid_constant__ BprepArgs pa) {
  extern __shared__ __align__(16) uint8_t bp_dyn[];
  __shared__ long long red[32];
  __shared__ long long s_r;
  __shared__ int s_meta[4];
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  bprep_seq<MAXB>(BlockSync(), pa, blockIdx.y, reinterpret_cast<uint2 *>(bp_dyn), red, &s_r, s_meta);
}

// ---------------------------------------------------------------------------
// k_bepi: per-(sequence, row) epilogue of a batched GEMM op
// ---------------------------------------------------------------------------
constexpr int BE_THREADS = 256;

__global__ void __launch_bounds__(BE_THREADS) k_bepi(const __grid_constant__ BepiArgs ea) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.y;
  const int u = blockIdx.x * BE_THREADS + threadIdx.x;
  const GemvArgs &a = ea.g;
  if (u < a.total_units) {
    const int si = seg_of(a, u);
    const BepiSeg &bs = ea.bs[si];
    GemvSeg sg = a.seg[si];
    const int row = u - sg.unit_begin;
    const size_t pstride = (size_t)ea.Bp * ea.ptot;
    const int64_t *pb = ea.p + (size_t)b * ea.ptot;
    long long p = 0, pu = 0;
    for (int s = 0; s < ea.S; ++s) p += pb[s * pstride + bs.p_row0 + row];
    const int e_x = ea.xmeta[2 * b], in_f = ea.xmeta[2 * b + 1];
    if (sg.out) sg.out = static_cast<uint8_t *>(sg.out) + b * bs.out_bs;
    if (sg.aux_out) sg.aux_out = static_cast<uint8_t *>(sg.aux_out) + b * bs.aux_bs;
    if (sg.p_out) sg.p_out = reinterpret_cast<int64_t *>(reinterpret_cast<uint8_t *>(sg.p_out) + b * bs.pout_bs);
    if (sg.mode == GM_SILU_MUL) {
      for (int s = 0; s < ea.S; ++s) pu += pb[s * pstride + bs.p_row0_up + row];
      epilogue_pair(a, sg, row, p << 4, pu << 4, e_x, in_f);
    } else {
      if (sg.mode == GM_CONV) {
        sg.aux0 = static_cast<uint8_t *>(sg.aux0) + b * bs.ring_bs;
        sg.T = &ea.params[b].T;
      }
      unsigned long long best = 0;
      epilogue_row(a, sg, row, p << 4, e_x, in_f, best);
    }
  }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
bool bgemm_tmap(TmapBytes *out, const uint8_t *w, int rows, int stride) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  static_assert(sizeof(CUtensorMap) == sizeof(TmapBytes), "CUtensorMap is 128 bytes");
  const cuuint64_t dims[2] = {(cuuint64_t)stride, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)stride};
  const cuuint32_t box[2] = {128, (cuuint32_t)BG_TILE};   // 2 groups x 128 rows, 128-byte swizzle
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = encode(reinterpret_cast<CUtensorMap *>(out), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                            const_cast<uint8_t *>(w), dims, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static cudaError_t launch_ex(const void *fn, void **args, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_bprep(const BprepArgs &a, cudaStream_t st, bool pdl) {
  if (a.K % 128 || a.K > 12288 || a.B < 1 || a.B > a.Bp) return cudaErrorInvalidValue;
  const int nblk = a.K / 8;
  const size_t xs_bytes = (size_t)((nblk + 127) / 128) * 4 * 32 * sizeof(uint2);
  void *args[] = {const_cast<BprepArgs *>(&a)};
  const int maxb = (nblk + BP_THREADS - 1) / BP_THREADS;
  const void *fn = maxb <= 1 ? (const void *)k_bprep<1> : maxb <= 2 ? (const void *)k_bprep<2> : (const void *)k_bprep<3>;
  return launch_ex(fn, args, dim3(1, a.B), dim3(BP_THREADS), xs_bytes, st, pdl);
}

size_t bgemm_smem(int Bp, int *ns) {
  const size_t stage = (size_t)BG_WBYTES + (size_t)Bp * 128 * BG_GPS;
  const size_t fixed = 1024;
  int n = (int)((BG_SMEM_MAX - fixed) / stage);
  if (n > BG_MAX_NS) n = BG_MAX_NS;
  if (ns) *ns = n;
  return fixed + (size_t)n * stage;
}

int bgemm_splits(int tiles, int NG, int ctas, bool argmax) {
  if (argmax) return 1;
  int best = 1;
  long long best_cost = -1;
  for (int s = 1; s <= NG; ++s) {
    if (NG % s || (NG / s) % 8) continue;
    const long long waves = ((long long)tiles * s + ctas - 1) / ctas;
    const long long cost = waves * (NG / s) * 16 + s;   // group-steps of the busiest CTA (+ split overhead)
    if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = s; }
  }
  return best;
}

template <int BP>
static cudaError_t launch_bg(const BgemmArgs &a, cudaStream_t st, bool pdl, int max_ctas) {
  int ns = 0;
  const size_t smem = bgemm_smem(BP, &ns);
  if (ns < 2) return cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_bgemm<BP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  BgemmArgs b = a;
  b.ns = ns;
  const int units = a.ntiles * a.S;
  const int grid = units < max_ctas ? units : max_ctas;
  void *args[] = {&b};
  return launch_ex((const void *)k_bgemm<BP>, args, dim3(grid), dim3(bg_threads(BP)), smem, st, pdl);
}

static unsigned long long *g_bg_trace = nullptr;   // process-wide trace buffer (f5_batch_trace)
unsigned long long *&bgemm_trace_buffer() { return g_bg_trace; }

cudaError_t launch_bgemm(BgemmArgs a, cudaStream_t st, bool pdl, int max_ctas) {
  if (!a.trace) a.trace = g_bg_trace;
  for (int i = 0; i < a.nseg; ++i)
    if ((reinterpret_cast<uintptr_t>(a.seg[i].w) & 15) || !bgemm_tmap(&a.tmap[i], a.seg[i].w, a.seg[i].rows, a.stride))
      return cudaErrorInvalidValue;
  if (a.K % 1024 || a.NG != a.K / 128 || a.S < 1 || a.NG % a.S || (a.NG / a.S) % 8 || a.ntiles < 1 ||
      a.B < 1 || a.B > a.Bp || a.stride % 16)
    return cudaErrorInvalidValue;
  switch (a.Bp) {
    case 16: return launch_bg<16>(a, st, pdl, max_ctas);
    case 32: return launch_bg<32>(a, st, pdl, max_ctas);
    case 64: return launch_bg<64>(a, st, pdl, max_ctas);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_bepi(const BepiArgs &a, cudaStream_t st, bool pdl) {
  if (a.g.total_units < 1) return cudaSuccess;
  void *args[] = {const_cast<BepiArgs *>(&a)};
  return launch_ex((const void *)k_bepi, args, dim3((a.g.total_units + BE_THREADS - 1) / BE_THREADS, a.B),
                   dim3(BE_THREADS), 0, st, pdl);
}

}  // namespace f5
