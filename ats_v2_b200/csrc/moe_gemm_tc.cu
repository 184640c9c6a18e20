// tcgen05 / TMEM grouped GEMMs for the bf16 SwiGLU experts (sm_100a).
//
// One persistent CTA per SM walks a static list of 128 x BN output tiles.
// Warp roles:
//   warp 0    TMA producer: 2-D tiled loads (128-byte swizzle) of the A and B
//             tiles into a 4-stage shared-memory ring, completion counted on
//             an mbarrier per stage.
//   warp 1    allocates 2*BN TMEM columns (two accumulators) and one thread
//             issues tcgen05.mma (M=128, N=BN, K=16, bf16 in, f32 accumulate)
//             four per 64-wide K block; tcgen05.commit frees each ring stage
//             and, after the last K block, hands the accumulator to the
//             epilogue.
//   warps 2-9 epilogue: two warps per 32-lane TMEM quadrant (= 32 tile rows),
//             each owning half of the tile's columns: tcgen05.ld, fused SwiGLU
//             forward / plain bf16 store / SwiGLU backward (whose pre-activation
//             loads are prefetched one 32-column chunk ahead), vector stores to
//             global; then release the accumulator, so the next tile's MMAs
//             overlap this tile's epilogue.
// Operands may be K-major or MN-major in shared memory (the tcgen05 descriptor
// says which), so every forward and backward GEMM of the experts reads its
// operands in place, without transposed copies:
//   M-grouped (forward, data gradients): tile rows are permuted token rows of
//     one expert segment; B is that expert's slice of the stacked weights.
//   K-grouped (weight gradients): the reduction runs over the expert's
//     segment rows; the output is that expert's weight gradient.
// Every wait is bounded (SM clock budget); a role that gives up records an
// error code in the plan's status word and raises a CTA-wide abort flag, the
// other roles stop, in-flight TMA loads and MMAs are drained, and TMEM is
// freed before the CTA exits.
#include <cudaTypedefs.h>

#include <mutex>

#include "moe_gemm.cuh"
#include "tc_ptx.cuh"

namespace ats {
namespace {

constexpr int BM = 128, BK = 64, STAGES = 4;
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, each owning half of the tile's columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr long long kWaitBudget = 4000000000LL;  // SM cycles, about 2 s

// Budget of the main-loop waits of this device's GEMM launches, read once per
// CTA.  ats_set_wait_budget shortens it so a test can make a wait run out; the
// drain waits, which make every issued TMA load and MMA finish before the CTA
// frees TMEM and exits, always keep the full kWaitBudget.
__device__ long long g_gemm_wait_budget = kWaitBudget;
// First GEMM wait on this device that gave up since the status was last taken
// (0: none).  The same code also goes to the call's own status word.
__device__ int g_gemm_status;
constexpr int kStageBox = 32 * 32 * 2;           // staging box: 32 rows x 32 bf16 columns, 64-byte swizzle
constexpr int kBoxesPerWarp = 2;
constexpr int kBandM = 16;  // M tiles per band of the tile order
constexpr int kMaxDevices = 64;

enum Epi { EPI_STORE = 0, EPI_SWIGLU_FWD = 1, EPI_SWIGLU_BWD = 2, EPI_F32 = 3, EPI_SCATTER = 4, EPI_ROPE = 5 };
constexpr int kMaxParts = 6;

// Where B (the stacked expert weights in M-grouped GEMMs) is read.
struct OpSpec {
  int group_rows;  // rows of one expert in the stacked weight
  int sub_offset;  // K-major B loaded as two halves, the second `sub_offset` rows further (0: one load)
};

struct GemmArgs {
  SegTable seg;  // segments of the permuted rows and their experts
  int M, N, K;   // M-grouped: N, K fixed; K-grouped: M, N fixed
  OpSpec b;
  bf16* out;  // output (bf16)
  int64_t ldo;
  int64_t out_group;  // K-grouped: elements between consecutive experts' outputs
  const bf16* h;      // SWIGLU_BWD: [rows, 2F] gate|up pre-activations
  bf16* h_out;        // SWIGLU_FWD: [rows, 2F]
  bf16* a_out;        // SWIGLU_FWD: [rows, F]
  int F;
  int* err;
  // Operand parts (SPLIT > 1): k block kb reads part kb % SPLIT, whose A tile starts a_koff
  // further along K, and whose B tile starts b_koff further along K and b_noff along N.  All
  // parts accumulate into one tile, so bf16 parts of a float32 operand give a float32 product.
  int a_koff[kMaxParts], b_koff[kMaxParts], b_noff[kMaxParts];
  float* out_f32;        // EPI_F32 output
  const float* bias;     // EPI_F32: added to every row (per column; may be null)
  int m_valid, n_valid;  // EPI_F32 / EPI_SCATTER: rows and columns of the output that exist
  const bf16* dxp;       // EPI_SCATTER: permuted-row gradients summed into each token (may be null)
  const int* tok_row;    // EPI_SCATTER: [T*topk] permuted row of (token, slot), -1 = dropped
  int topk;
  const bf16* rope_cos;  // EPI_ROPE: [rope_seq, 128] cos and sin tables; row r of the output is position
  const bf16* rope_sin;  //   r % rope_seq (rows are [batch, seq] flattened)
  int rope_seq;
};

// tile -> (group, weight index, m tile, n tile, k blocks).  Groups are the
// segments (M-grouped) or the experts (K-grouped), scanned linearly.
struct TileInfo {
  int g, e, mt, nt, kb;
};

// N tiles of a group.  N need not be a multiple of BN for the plain store: the last tile's columns past N read
// zero-filled B tiles and are not stored.
template <int BN, bool KGROUP, int EPI>
__device__ __forceinline__ int n_tiles(const GemmArgs& p) {
  return EPI == EPI_SWIGLU_FWD ? p.F / (BN / 2) : (p.N + BN - 1) / BN;
}

template <bool KGROUP>
__device__ __forceinline__ int n_groups(const GemmArgs& p) {
  return KGROUP ? p.seg.E : p.seg.nseg;
}

// Tiles of group g: its M tiles (TM rows: 128, or 256 for a CTA pair, whose last tile may have only its first
// 128-row half inside the group) times the N tiles.
template <int BN, bool KGROUP, int EPI, int TM>
__device__ __forceinline__ int group_tiles(const GemmArgs& p, int g) {
  return ((KGROUP ? p.M : p.seg.rows[g]) + TM - 1) / TM * n_tiles<BN, KGROUP, EPI>(p);
}

// Rows a K-grouped GEMM reduces over in segment s: its kept rows rounded up to one K block (the rest of the
// segment is zero padding), or all its rows when the table has no kept counts.
__device__ __forceinline__ int seg_krows(const SegTable& sg, int s) {
  const int r = sg.rows[s];
  if (sg.kept == nullptr) return r;
  const int k = (sg.kept[s] + BK - 1) / BK * BK;
  return k < 0 ? 0 : (k < r ? k : r);
}

// Walks the groups in order: a role visits its tiles t = blockIdx.x + i*gridDim.x in increasing order,
// so a cursor (group, first tile of the group) that only moves forward decodes every tile.
struct TileCursor {
  int g = 0, first = 0;
};

template <int BN, bool KGROUP, int EPI, int SPLIT, int TM>
__device__ __forceinline__ void decode_tile(const GemmArgs& p, TileCursor& cur, int t, TileInfo& ti) {
  const int NT = n_tiles<BN, KGROUP, EPI>(p);
  int n = group_tiles<BN, KGROUP, EPI, TM>(p, cur.g);
  while (t >= cur.first + n) {  // t < total, so a later group holds it
    cur.first += n;
    ++cur.g;
    n = group_tiles<BN, KGROUP, EPI, TM>(p, cur.g);
  }
  const int g = cur.g;
  const int q = t - cur.first;
  ti.g = g;
  // bands of kBandM M tiles, M fastest inside a band: the CTAs that run together share their B tiles
  // and the band's A rows, so both stay in L2 even when a weight is larger than L2
  const int MT = n / NT;
  const int band = q / (kBandM * NT);
  const int m0 = band * kBandM;
  const int gm = MT - m0 < kBandM ? MT - m0 : kBandM;
  const int r = q - band * kBandM * NT;
  ti.nt = r / gm;
  ti.mt = m0 + (r - ti.nt * gm);
  if (KGROUP) {
    ti.e = g;
    int kb = 0;
    for (int u = 0; u < p.seg.spe; ++u) kb += seg_krows(p.seg, p.seg.eseg[g * p.seg.spe + u]) / BK;
    ti.kb = kb * SPLIT;
  } else {
    ti.e = p.seg.expert[g];
    ti.kb = (p.K / BK) * SPLIT;
  }
}

// Shared memory of the epilogue's staging boxes: the bf16-output epilogues write through them.
__host__ __device__ constexpr int staging_bytes(int epi) {
  return (epi == EPI_STORE || epi == EPI_SWIGLU_FWD || epi == EPI_SWIGLU_BWD || epi == EPI_SCATTER ||
          epi == EPI_ROPE)
             ? kEpiWarps * kBoxesPerWarp * kStageBox
             : 0;
}

// Ring of a launch: one A tile (128 x 64) and BPARTS B tiles per stage; a CTA of a pair holds half of the
// B rows.  Every launch fills the same 224 KB, less its epilogue's staging boxes, with as many stages as
// fit (4 for 128 x 256 tiles, 6 for 128 x 128 tiles or pair halves, 5 for the float32 router tiles, which
// stage nothing): the GEMMs wait on load latency, and more bytes in flight hide more of it.
constexpr int kRingBytes = STAGES * (BM * BK * 2 + 256 * BK * 2);
__host__ __device__ constexpr int stage_bytes(int bn, int bparts, bool pair) {
  return BM * BK * 2 + bparts * (pair ? bn / 2 : bn) * BK * 2;
}
__host__ __device__ constexpr int ring_stages(int bn, int bparts, bool pair, int epi) {
  return (kRingBytes + kEpiWarps * kBoxesPerWarp * kStageBox - staging_bytes(epi)) / stage_bytes(bn, bparts, pair);
}

// One epilogue warp's bf16 output path: a 32 x 32 chunk (row = lane, 32 packed bf16 pairs per lane
// in pk[16]) goes into the next of the warp's staging boxes in the 64-byte swizzled layout, then out
// with one TMA store, so global writes are whole lines and asynchronous.  A box is reused once the
// store that last read it is done reading.
struct BoxWriter {
  uint8_t* base;  // this warp's kBoxesPerWarp boxes
  int n;          // stores issued
  __device__ __forceinline__ void put(const uint32_t (&pk)[16], const CUtensorMap* map, int x, int y, int lane) {
    uint8_t* box = base + (n % kBoxesPerWarp) * kStageBox;
    if (lane == 0) tc::bulk_wait_read<kBoxesPerWarp - 1>();
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // row `lane`, 16-byte chunk q at its swizzled place (conflict-free)
      uint4* d = reinterpret_cast<uint4*>(box + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4));
      *d = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    }
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tc::tma_store_2d(map, box, x, y);
      tc::bulk_commit();
    }
    ++n;
  }
};

__device__ __forceinline__ void fail_abort(int* err, volatile int* abort, int code) {
  if (*abort == 0) {
    *abort = 1;
    atomicCAS(err, 0, code);
    atomicCAS(&g_gemm_status, 0, code);
  }
}

__device__ __forceinline__ void fail_drain(int* err, int code) {
  atomicCAS(err, 0, code);
  atomicCAS(&g_gemm_status, 0, code);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void pack32(const float (&v)[32], uint32_t (&pk)[16]) {
#pragma unroll
  for (int q = 0; q < 16; ++q) pk[q] = pack_bf16(v[2 * q], v[2 * q + 1]);
}

__device__ __forceinline__ void load32(const bf16* src, float (&v)[32]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w = s[q];
    const bf16* e = reinterpret_cast<const bf16*>(&w);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[q * 8 + i] = __bfloat162float(e[i]);
  }
}

// PAIR: a cluster of two CTAs on two SMs computes each 256 x BN tile with cta_group::2 MMAs.  CTA r of the
// pair loads rows [128 r, 128 r + 128) of the tile's A and rows [r BN/2, (r + 1) BN/2) of its B (the D
// columns; for the SwiGLU forward the gate rows in CTA 0 and the up rows in CTA 1), each into its own
// ring, so a CTA reads half the B bytes of a single-CTA 128 x BN tile for the same MMA work and the ring
// holds more stages.  Both CTAs' loads of a stage complete on CTA 0's full barrier, which CTA 0's producer
// arms for both halves; CTA 0's MMA thread waits on it alone.  CTA 0's MMA commits free the stage and hand
// over the accumulator on both CTAs' barriers; both CTAs' epilogues (each its 128 rows, all BN columns, in
// its own TMEM) release the accumulator on CTA 0's barrier.  A tile whose second half lies past the group
// is computed whole, its second half not stored.  At the end the CTAs meet at a cluster barrier; CTA 0
// then settles the stages that only one producer reached (a role gave up) and waits until every load of
// both CTAs has landed; a second cluster barrier keeps CTA 1 alive until then.
template <int BN, bool A_MN, bool B_MN, int EPI, bool KGROUP, int SPLIT, int BPARTS, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                              const __grid_constant__ CUtensorMap tmB,
                                                              const __grid_constant__ CUtensorMap tmO,
                                                              const __grid_constant__ CUtensorMap tmO2,
                                                              GemmArgs p) {
  constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of a B tile (columns of D) held by this CTA
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = B_ROWS * BK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + BPARTS * B_BYTES;  // one A tile, BPARTS B tiles
  static_assert(STAGE_BYTES == (uint32_t)stage_bytes(BN, BPARTS, PAIR), "stage layout");
  constexpr int NST = ring_stages(BN, BPARTS, PAIR, EPI);
  constexpr int TM = PAIR ? 2 * BM : BM;  // rows of an output tile
  static_assert(SPLIT == 1 || BPARTS == 1, "operand parts along K or in the stage, not both");
  static_assert(!PAIR || (SPLIT == 1 && BPARTS == 1 && (BN == 128 || BN == 256) &&
                          (EPI == EPI_STORE || EPI == EPI_SWIGLU_FWD || EPI == EPI_SWIGLU_BWD)),
                "CTA pairs run the plain, SwiGLU-forward and SwiGLU-backward expert GEMMs");
  constexpr uint32_t IDESC = tc::idesc_bf16(TM, BN, A_MN, B_MN);
  extern __shared__ uint8_t smem_raw[];
  // dynamic shared memory: the 1024-byte aligned ring (the 128-byte swizzle atom spans 1024 bytes),
  // the epilogue's store staging (EPI_STORE: one 2 KB 32 x 32 bf16 box per epilogue warp), then the
  // per-group tile prefix
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = ring + NST * STAGE_BYTES;
  __shared__ __align__(8) uint64_t full_bar[NST], empty_bar[NST], tfull_bar[2], tempty_bar[2], done_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int peer_issued_s;  // PAIR, CTA 0: stages CTA 1's producer loaded
  __shared__ int total_s;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long budget = g_gemm_wait_budget;
  const uint32_t cta = PAIR ? tc::cluster_ctarank() : 0u;  // this CTA's half of a pair tile
  const int t_first = PAIR ? (int)tc::cluster_id_x() : (int)blockIdx.x;
  const int t_step = PAIR ? (int)tc::ncluster_x() : (int)gridDim.x;
  // a role that gives up stops the other roles of this CTA and, in a pair, of the other CTA
  auto give_up = [&](int code) {
    fail_abort(p.seg.err, &abort_flag, code);
    if constexpr (PAIR) tc::st_cluster_u32(tc::cluster_addr(tc::smem_u32((const void*)&abort_flag), cta ^ 1u), 1u);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(&full_bar[s], 1);
      tc::mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&tfull_bar[a], 1);
      tc::mbar_init(&tempty_bar[a], PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    tc::mbar_init(&done_bar, 1);
    tc::fence_barrier_init();
    tc::fence_proxy_async_smem();
    abort_flag = 0;
    int total = 0;
    for (int g = 0; g < n_groups<KGROUP>(p); ++g) total += group_tiles<BN, KGROUP, EPI, TM>(p, g);
    total_s = total;
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tc::tmem_alloc_pair(&tmem_base_s, 2 * BN);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(&tmem_base_s, 2 * BN);
      tc::tmem_relinquish();
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) tc::cluster_sync();  // both CTAs' barriers exist before either signals the other's
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  const int total = total_s;
  // every load issued lands before the CTA may exit: wait for the last phase of each stage used by the
  // first `issued` stage loads (phases of a stage complete in order)
  auto drain_loads = [&](int issued) {
    for (int s = 0; s < NST && s < issued; ++s) {
      const int klast = s + (issued - 1 - s) / NST * NST;
      if (!tc::mbar_wait(&full_bar[s], (uint32_t)((klast / NST) & 1), nullptr, kWaitBudget))
        fail_drain(p.seg.err, 11);
    }
  };
  int issued_k = 0;  // producer: stage loads issued

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tc::prefetch_tensormap(&tmA);
      tc::prefetch_tensormap(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      // a pair's loads count on CTA 0's full barriers
      const uint32_t full0 = PAIR ? tc::cluster_addr(tc::smem_u32(&full_bar[0]), 0u) : 0u;
      auto load = [&](void* dst, const CUtensorMap* map, int x, int y) {
        if constexpr (PAIR)
          tc::tma_load_2d_pair(dst, map, x, y, full0 + (uint32_t)stage * 8u);
        else
          tc::tma_load_2d(dst, map, x, y, &full_bar[stage]);
      };
      // MN-major operands: one load of `blocks` 64-column blocks of 64 K rows (a 3-D map: 64 columns, the K
      // rows, the column blocks), each block 8 KB in shared memory -- the layout of that many 2-D 64 x 64
      // boxes in one TMA instruction instead of one per block
      auto load_mn = [&](void* dst, const CUtensorMap* map, int col, int krow) {
        if constexpr (PAIR)
          tc::tma_load_3d_pair(dst, map, 0, krow, col >> 6, full0 + (uint32_t)stage * 8u);
        else
          tc::tma_load_3d(dst, map, 0, krow, col >> 6, &full_bar[stage]);
      };
      TileCursor cur;
      for (int t = t_first; t < total && !abort_flag; t += t_step) {
        TileInfo ti;
        decode_tile<BN, KGROUP, EPI, SPLIT, TM>(p, cur, t, ti);
        const int m0 = ti.mt * TM + (int)cta * BM;
        const int n0 = EPI == EPI_SWIGLU_FWD ? ti.nt * (BN / 2) : ti.nt * BN;
        // K blocks: M-grouped = kb of the fixed K; K-grouped = the expert's segments' rows, in order.
        // The segment's first row and k-block count live in registers; the table is read only
        // when the walk moves to the next segment.
        int u = 0, lkb = 0;
        int seg_kb = 0, seg_r0 = KGROUP ? 0 : p.seg.row0[ti.g];
        if (KGROUP) {
          const int s0 = p.seg.eseg[ti.g * p.seg.spe];
          seg_kb = seg_krows(p.seg, s0) / BK;
          seg_r0 = p.seg.row0[s0];
        }
        const int b_row0 = ti.e * p.b.group_rows;
        for (int kb = 0; kb < ti.kb; ++kb) {
          const int part = SPLIT == 1 ? 0 : kb % SPLIT;
          const int kq = SPLIT == 1 ? kb : kb / SPLIT;  // K block of the fixed-K (M-grouped) loop
          const int a_ko = SPLIT == 1 ? 0 : p.a_koff[part];
          const int b_ko = SPLIT == 1 ? 0 : p.b_koff[part];
          const int b_no = SPLIT == 1 ? 0 : p.b_noff[part];
          if (KGROUP && part == 0) {
            while (lkb >= seg_kb) {  // next non-empty segment of this expert
              ++u;
              lkb = 0;
              const int sn = p.seg.eseg[ti.g * p.seg.spe + u];
              seg_kb = seg_krows(p.seg, sn) / BK;
              seg_r0 = p.seg.row0[sn];
            }
          }
          if (!tc::mbar_wait(&empty_bar[stage], phase ^ 1u, &abort_flag, budget)) {
            give_up(1);
            break;
          }
          uint8_t* sa = ring + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          if (cta == 0) tc::mbar_arrive_expect_tx(&full_bar[stage], PAIR ? 2 * STAGE_BYTES : STAGE_BYTES);
          if (!A_MN) {  // M-grouped A: rows of the tile's segment, K contiguous
            load(sa, &tmA, a_ko + kq * BK, seg_r0 + m0);
          } else {      // K-grouped A: M contiguous, K = rows of the current segment
            load_mn(sa, &tmA, m0, seg_r0 + lkb * BK + a_ko);
          }
          if (!B_MN) {  // stacked weights, K contiguous
            if constexpr (PAIR) {  // this CTA's B_ROWS rows: the gate or up half (SwiGLU), or the cta-th half
              const int brow = b_row0 + n0 + (p.b.sub_offset ? (cta ? p.b.sub_offset : 0) : (int)cta * B_ROWS);
              load(sb, &tmB, kq * BK, brow);
            } else if constexpr (BPARTS > 1) {  // the parts are consecutive rows: one box holds them all
              load(sb, &tmB, b_ko + kq * BK, b_row0 + n0 + b_no);
            } else {
              const int brow = b_row0 + n0 + b_no;
              load(sb, &tmB, b_ko + kq * BK, brow);
              if (p.b.sub_offset) load(sb + (BN / 2) * 128, &tmB, b_ko + kq * BK, brow + p.b.sub_offset);
            }
          } else {
            const int krow = (KGROUP ? seg_r0 + lkb * BK : b_row0 + kq * BK) + b_ko;
            const int ncol = n0 + (int)cta * B_ROWS + b_no;
            load_mn(sb, &tmB, ncol, krow);  // B_ROWS / 64 blocks per part, the parts consecutive: one load
          }
          if (part == SPLIT - 1) ++lkb;
          ++issued_k;
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if constexpr (PAIR) {  // CTA 0 drains both CTAs' loads after the first cluster barrier
        if (cta != 0) tc::st_cluster_u32(tc::cluster_addr(tc::smem_u32(&peer_issued_s), 0u), (uint32_t)issued_k);
      } else {
        drain_loads(issued_k);
      }
    }
  } else if (warp == 1) {
    if ((!PAIR || cta == 0) && lane == 0) {
      // ---------------------------------------------------------------- MMA
      int stage = 0;
      uint32_t phase = 0;
      int i = 0;
      bool issued = false;
      const uint32_t a_lbo = A_MN ? 8192u : 16u, b_lbo = B_MN ? 8192u : 16u;
      const uint32_t a_step = A_MN ? 2048u : 32u, b_step = B_MN ? 2048u : 32u;
      // a pair's commits arrive on the barrier of each CTA (this CTA's address, then the other's)
      auto commit = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          tc::mma_commit_pair(tc::cluster_addr(tc::smem_u32(bar), 0u));
          tc::mma_commit_pair(tc::cluster_addr(tc::smem_u32(bar), 1u));
        } else {
          tc::mma_commit(bar);
        }
      };
      TileCursor cur;
      for (int t = t_first; t < total && !abort_flag; t += t_step, ++i) {
        TileInfo ti;
        decode_tile<BN, KGROUP, EPI, SPLIT, TM>(p, cur, t, ti);
        const int acc = i & 1;
        const uint32_t acc_phase = (uint32_t)(i >> 1) & 1u;
        if (!tc::mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, &abort_flag, budget)) {
          give_up(2);
          break;
        }
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < ti.kb; ++kb) {
          if (!tc::mbar_wait(&full_bar[stage], phase, &abort_flag, budget)) {
            give_up(3);
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sa = tc::smem_u32(ring + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = tc::smem_desc(sa + k * a_step, a_lbo, 1024u, tc::kLayoutSW128);
#pragma unroll
            for (int j = 0; j < BPARTS; ++j) {  // the B parts of the stage share the A tile
              const uint64_t bd = tc::smem_desc(sb + j * B_BYTES + k * b_step, b_lbo, 1024u, tc::kLayoutSW128);
              if constexpr (PAIR)
                tc::mma_bf16_pair(d_tmem, ad, bd, IDESC, (kb > 0 || k > 0 || j > 0) ? 1u : 0u);
              else
                tc::mma_bf16(d_tmem, ad, bd, IDESC, (kb > 0 || k > 0 || j > 0) ? 1u : 0u);
            }
          }
          commit(&empty_bar[stage]);
          issued = true;
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (ti.kb > 0) {
          commit(&tfull_bar[acc]);
        } else {  // no K blocks (an expert without rows): the epilogue writes zeros
          tc::mbar_arrive(&tfull_bar[acc]);
          if constexpr (PAIR) tc::mbar_arrive_cluster(tc::cluster_addr(tc::smem_u32(&tfull_bar[acc]), 1u));
        }
      }
      // drain: all issued MMAs complete before TMEM may be freed
      if (issued) {
        if constexpr (PAIR)
          tc::mma_commit_pair(tc::cluster_addr(tc::smem_u32(&done_bar), 0u));
        else
          tc::mma_commit(&done_bar);
        if (!tc::mbar_wait(&done_bar, 0u, nullptr, kWaitBudget)) fail_drain(p.seg.err, 12);
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int quad = warp & 3;         // TMEM lanes [32*quad, 32*quad + 32)
    const int chalf = (warp - 2) >> 2;  // which half of the tile's columns
    const int row_in_tile = quad * 32 + lane;
    BoxWriter bw{staging + (warp - 2) * kBoxesPerWarp * kStageBox, 0};
    int i = 0;
    TileCursor cur;
    for (int t = t_first; t < total && !abort_flag; t += t_step, ++i) {
      TileInfo ti;
      decode_tile<BN, KGROUP, EPI, SPLIT, TM>(p, cur, t, ti);
      const int acc = i & 1;
      const uint32_t acc_phase = (uint32_t)(i >> 1) & 1u;
      // first row of this CTA's 128 rows in the group; a pair tile's second half may lie past the group's
      // rows (it is computed with whatever the loads brought and not stored)
      const int mrow = ti.mt * TM + (int)cta * BM;
      const bool half_ok = !PAIR || mrow < (KGROUP ? p.M : p.seg.rows[ti.g]);
      if constexpr (EPI == EPI_SWIGLU_BWD) {
        // the pre-activations do not depend on the accumulator: start loading them now
        const int64_t row = (int64_t)p.seg.row0[ti.g] + mrow + row_in_tile;
        const int64_t F2 = 2 * (int64_t)p.F;
        const int c0 = chalf * (BN / 2);
        const bf16* hg = p.h + row * F2 + ti.nt * BN + c0;
        const bf16* hu = hg + p.F;
        uint4 gq[4], uq[4];
        if (half_ok) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            gq[q] = reinterpret_cast<const uint4*>(hg)[q];
            uq[q] = reinterpret_cast<const uint4*>(hu)[q];
          }
        }
        if (!tc::mbar_wait(&tfull_bar[acc], acc_phase, &abort_flag, budget)) {
          give_up(4);
          break;
        }
        tc::tc_fence_after();
        const uint32_t t_row = tmem_base + (uint32_t)(acc * BN + c0) + ((uint32_t)(quad * 32) << 16);
        const int row_base = p.seg.row0[ti.g] + mrow + quad * 32;
        const int x0 = ti.nt * BN + c0;
#pragma unroll 1
        for (int c = 0; c < (half_ok ? BN / 2 : 0); c += 32) {
          float dv[32];
          tc::tmem_ld32(t_row + c, dv);
          // column pairs: word i of a chunk holds columns 2i (low half) and 2i+1
          uint32_t g2[16], u2[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            g2[4 * q] = gq[q].x, g2[4 * q + 1] = gq[q].y, g2[4 * q + 2] = gq[q].z, g2[4 * q + 3] = gq[q].w;
            u2[4 * q] = uq[q].x, u2[4 * q + 1] = uq[q].y, u2[4 * q + 2] = uq[q].z, u2[4 * q + 3] = uq[q].w;
          }
          if (c + 32 < BN / 2) {  // prefetch the next chunk while this one computes
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              gq[q] = reinterpret_cast<const uint4*>(hg + c + 32)[q];
              uq[q] = reinterpret_cast<const uint4*>(hu + c + 32)[q];
            }
          }
          uint32_t pkg[16], pku[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            swiglu_grad_bf2(g2[i], u2[i], bf2_pack(dv[2 * i], dv[2 * i + 1]), pkg[i], pku[i]);
          bw.put(pkg, &tmO, x0 + c, row_base, lane);        // dg into dh[:, :F]
          bw.put(pku, &tmO, p.F + x0 + c, row_base, lane);  // du into dh[:, F:]
        }
      } else if constexpr (EPI == EPI_SCATTER) {
        // token gradient: the router's share (this tile, cast to bf16) plus the token's kept
        // permuted-row gradients summed in ascending row (= expert) order, as two bf16 gradients add.
        // The row gradients do not depend on the accumulator: the first kPre kept rows' first chunk
        // loads before the accumulator wait, and each next chunk while the current one is summed.
        constexpr int kPre = 2;
        const int c0 = chalf * (BN / 2);
        const int64_t tok = (int64_t)p.seg.row0[ti.g] + mrow + row_in_tile;
        const bool ok = tok < p.m_valid;
        int rows[kMaxTopK];
        int n = 0;
        if (ok && p.dxp != nullptr) {
          for (int s2 = 0; s2 < p.topk; ++s2) {
            const int r = p.tok_row[tok * p.topk + s2];
            if (r < 0) continue;
            int q = n++;
            while (q > 0 && rows[q - 1] > r) {
              rows[q] = rows[q - 1];
              --q;
            }
            rows[q] = r;
          }
        }
        const int npre = n < kPre ? n : kPre;
        const int64_t col_base = (int64_t)ti.nt * BN + c0;
        const int row_base = p.seg.row0[ti.g] + mrow + quad * 32;  // rows at or past T are clipped
        const bf16* prow[kPre];
#pragma unroll
        for (int r = 0; r < kPre; ++r) prow[r] = p.dxp + (int64_t)(r < npre ? rows[r] : 0) * p.ldo + col_base;
        uint4 pre[kPre][4];
#pragma unroll
        for (int r = 0; r < kPre; ++r)
          if (r < npre) {
            const uint4* src = reinterpret_cast<const uint4*>(prow[r]);
#pragma unroll
            for (int q = 0; q < 4; ++q) pre[r][q] = src[q];
          }
        if (!tc::mbar_wait(&tfull_bar[acc], acc_phase, &abort_flag, budget)) {
          give_up(4);
          break;
        }
        tc::tc_fence_after();
        const uint32_t t_row = tmem_base + (uint32_t)(acc * BN) + ((uint32_t)(quad * 32) << 16);
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          float v[32];
          tc::tmem_ld32(t_row + c0 + c, v);
          uint4 cur[kPre][4];
#pragma unroll
          for (int r = 0; r < kPre; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) cur[r][q] = pre[r][q];
          if (c + 32 < BN / 2) {
#pragma unroll
            for (int r = 0; r < kPre; ++r)
              if (r < npre) {
                const uint4* src = reinterpret_cast<const uint4*>(prow[r] + c + 32);
#pragma unroll
                for (int q = 0; q < 4; ++q) pre[r][q] = src[q];
              }
          }
          if (ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = round_to<bf16>(v[j]);
            if (n > 0) {
              float m[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) m[j] = 0.f;
#pragma unroll
              for (int r = 0; r < kPre; ++r)
                if (r < npre) {
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const bf16* e = reinterpret_cast<const bf16*>(&cur[r][q]);
#pragma unroll
                    for (int i2 = 0; i2 < 8; ++i2) m[q * 8 + i2] += __bfloat162float(e[i2]);
                  }
                }
              for (int i2 = kPre; i2 < n; ++i2) {  // more than kPre kept experts: loaded in place
                float u[32];
                load32(p.dxp + (int64_t)rows[i2] * p.ldo + col_base + c, u);
#pragma unroll
                for (int j = 0; j < 32; ++j) m[j] += u[j];
              }
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(round_to<bf16>(m[j]), v[j]);
            }
          }
          uint32_t pk[16];
          pack32(v, pk);
          bw.put(pk, &tmO, (int)(col_base + c), row_base, lane);
        }
      } else {
        if (!tc::mbar_wait(&tfull_bar[acc], acc_phase, &abort_flag, budget)) {
          give_up(4);
          break;
        }
        tc::tc_fence_after();
        const uint32_t t_row = tmem_base + (uint32_t)(acc * BN) + ((uint32_t)(quad * 32) << 16);
        if (!half_ok) {
          // the half of a pair tile past the group: nothing to store
        } else if constexpr (EPI == EPI_SWIGLU_FWD) {
          const int c0 = chalf * (BN / 4);
          const int n0 = ti.nt * (BN / 2) + c0;
          const int row_base = p.seg.row0[ti.g] + mrow + quad * 32;
#pragma unroll 1
          for (int c = 0; c < BN / 4; c += 32) {
            float gv[32], uv[32];
            tc::tmem_ld32(t_row + c0 + c, gv);
            tc::tmem_ld32(t_row + BN / 2 + c0 + c, uv);
            uint32_t pg[16], pu[16], pa[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {  // h rounded to bf16 once; a from those rounded values
              pg[i] = bf2_pack(gv[2 * i], gv[2 * i + 1]);
              pu[i] = bf2_pack(uv[2 * i], uv[2 * i + 1]);
              pa[i] = silu_mul_bf2(pg[i], pu[i]);
            }
            bw.put(pg, &tmO, n0 + c, row_base, lane);        // gate half of h
            bw.put(pu, &tmO, p.F + n0 + c, row_base, lane);  // up half of h
            bw.put(pa, &tmO2, n0 + c, row_base, lane);       // a
          }
        } else if constexpr (EPI == EPI_F32) {
          // float32 tile, rows below m_valid and columns below n_valid, plus a per-column bias
          const bool zero = ti.kb == 0;
          const int c0 = chalf * (BN / 2);
          const int64_t row = KGROUP ? (int64_t)mrow + row_in_tile
                                     : (int64_t)p.seg.row0[ti.g] + mrow + row_in_tile;
          float* outp = p.out_f32 + (KGROUP ? (int64_t)ti.e * p.out_group : 0) + row * p.ldo;
          const bool vec4 = (p.ldo & 3) == 0;
#pragma unroll 1
          for (int c = 0; c < BN / 2; c += 32) {
            float v[32];
            if (!zero) {
              tc::tmem_ld32(t_row + c0 + c, v);  // warp-wide: every lane loads, stores are guarded
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.f;
            }
            const int col0 = ti.nt * BN + c0 + c;
            if (row < p.m_valid) {
              if (p.bias != nullptr) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < p.n_valid) v[j] = __fadd_rn(v[j], p.bias[col0 + j]);
              }
              if (vec4 && col0 + 32 <= p.n_valid) {
                float4* d = reinterpret_cast<float4*>(outp + col0);
#pragma unroll
                for (int q = 0; q < 8; ++q) d[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < p.n_valid) outp[col0 + j] = v[j];
              }
            }
          }
        } else if constexpr (EPI == EPI_ROPE) {
          // one head of 128 dims per tile (BN = 128).  The warp of column half `chalf` takes the column
          // pairs (d, d + 64), d in [32*chalf, 32*chalf + 32), which rotate-half mixes:
          //   out[d]      = q[d]*cos[d]           - q[d+64]*sin[d]
          //   out[d + 64] = q[d+64]*cos[d+64]     + q[d]*sin[d+64]
          // q is the GEMM result rounded to bf16; each product and the sum round to bf16, as the bf16
          // torch operations of apply_rotary_pos_emb round them (ats/model/rope.py:83-86)
          const int d0 = chalf * 32;
          const int64_t tok = (int64_t)p.seg.row0[ti.g] + mrow + row_in_tile;
          const int64_t pos = tok < p.m_valid ? tok % p.rope_seq : 0;  // rows past the end are clipped
          float q1[32], q2[32];
          tc::tmem_ld32(t_row + d0, q1);
          tc::tmem_ld32(t_row + 64 + d0, q2);
          const uint4* cs1 = reinterpret_cast<const uint4*>(p.rope_cos + pos * 128 + d0);
          const uint4* cs2 = reinterpret_cast<const uint4*>(p.rope_cos + pos * 128 + 64 + d0);
          const uint4* sn1 = reinterpret_cast<const uint4*>(p.rope_sin + pos * 128 + d0);
          const uint4* sn2 = reinterpret_cast<const uint4*>(p.rope_sin + pos * 128 + 64 + d0);
          uint32_t o1[16], o2[16];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint4 c1 = cs1[q4], c2 = cs2[q4], s1 = sn1[q4], s2 = sn2[q4];
            const uint32_t cw1[4] = {c1.x, c1.y, c1.z, c1.w}, cw2[4] = {c2.x, c2.y, c2.z, c2.w};
            const uint32_t sw1[4] = {s1.x, s1.y, s1.z, s1.w}, sw2[4] = {s2.x, s2.y, s2.z, s2.w};
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const int i = 4 * q4 + kk;
              const uint32_t a = bf2_pack(q1[2 * i], q1[2 * i + 1]), b = bf2_pack(q2[2 * i], q2[2 * i + 1]);
              o1[i] = bf2_add(bf2_mul(a, cw1[kk]), bf2_mul(b ^ 0x80008000u, sw1[kk]));  // rotate_half: -q[d+64]
              o2[i] = bf2_add(bf2_mul(b, cw2[kk]), bf2_mul(a, sw2[kk]));
            }
          }
          const int row_base = p.seg.row0[ti.g] + mrow + quad * 32;
          bw.put(o1, &tmO, ti.nt * 128 + d0, row_base, lane);
          bw.put(o2, &tmO, ti.nt * 128 + 64 + d0, row_base, lane);
        } else {
          // plain bf16 store: each 32 x 32 chunk (this warp's 32 rows) goes through shared memory in
          // the 64-byte swizzled layout and out with one TMA store, so global writes are whole lines
          const bool zero = ti.kb == 0;
          const int c0 = chalf * (BN / 2);
          // first of this warp's rows in the output map: [E][M] stacked weight rows, or the permuted rows
          const int row_base = (KGROUP ? ti.e * p.M : p.seg.row0[ti.g]) + mrow + quad * 32;
#pragma unroll 1
          for (int c = 0; c < BN / 2; c += 32) {
            if (ti.nt * BN + c0 + c >= p.N) break;  // a chunk past N (the last tile of an N not a multiple of BN)
            float v[32];
            if (!zero) {
              tc::tmem_ld32(t_row + c0 + c, v);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.f;
            }
            uint32_t pk[16];
            pack32(v, pk);
            bw.put(pk, &tmO, ti.nt * BN + c0 + c, row_base, lane);
          }
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {  // the accumulator is free again (a pair's MMA thread counts both CTAs' warps)
        if (PAIR && cta != 0)
          tc::mbar_arrive_cluster(tc::cluster_addr(tc::smem_u32(&tempty_bar[acc]), 0u));
        else
          tc::mbar_arrive(&tempty_bar[acc]);
      }
    }
    if (staging_bytes(EPI) > 0 && lane == 0) tc::bulk_wait<0>();  // every TMA store done before the CTA exits
  }
  tc::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) {
    // CTA 0's MMAs read CTA 1's ring and write its TMEM, and CTA 1's loads and epilogue signal CTA 0's
    // barriers: after the first barrier CTA 0 knows how many stages each producer loaded.  Where only one
    // of them loaded a stage (the other gave up), CTA 0 settles that stage's transaction count -- the
    // missing half counted as done, or the half on its way expected -- and then waits for every phase, so
    // no load of either CTA is in flight when the second barrier lets them free TMEM and exit.
    tc::cluster_sync();
    if (cta == 0 && warp == 0 && lane == 0) {
      const int kl = issued_k, kp = peer_issued_s;
      const int lo = kl < kp ? kl : kp, hi = kl < kp ? kp : kl;
      if (hi - lo > NST) {  // cannot happen: a stage is reloaded only after both halves of its last load
        fail_drain(p.seg.err, 13);
      } else {
        for (int k = lo; k < hi; ++k) {
          if (k < kl)
            tc::mbar_complete_tx(&full_bar[k % NST], STAGE_BYTES);  // CTA 1's half never came
          else
            tc::mbar_arrive_expect_tx(&full_bar[k % NST], STAGE_BYTES);  // only CTA 1's half is coming
        }
        drain_loads(hi);
      }
    }
    tc::cluster_sync();
  }
  if (warp == 1) {
    tc::tc_fence_after();
    if constexpr (PAIR)
      tc::tmem_dealloc_pair(tmem_base, 2 * BN);
    else
      tc::tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ------------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int encode_fn(PFN_cuTensorMapEncodeTiled_v12000* out) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return fail(ATS_ECUDA, "moe_gemm: cuTensorMapEncodeTiled unavailable");
  *out = g_encode;
  return ATS_OK;
}

// 2-D bf16 tensor map, inner dim contiguous, box {box_inner, box_outer}.
int encode_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
               uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  ATS_TRY(encode_fn(&enc));
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15) || inner < box_inner || outer < box_outer)
    return fail(ATS_EBADARG, "moe_gemm: operand not TMA-compatible (base %p, row %llu B, %llu x %llu)", base,
                (unsigned long long)row_bytes, (unsigned long long)inner, (unsigned long long)outer);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ATS_ECUDA, "moe_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return ATS_OK;
}

// MN-major operand map: the 2-D tensor [outer rows][inner] (inner a multiple of 64) seen in three dimensions
// {64 columns, the rows, inner / 64 column blocks} with strides {row_bytes, 128 B}, 128-byte swizzle, box
// {64, 64, blocks}: one load brings `blocks` consecutive 64 x 64 blocks, block-major in shared memory.  Blocks
// and rows past the tensor read as zeros.
int make_map_mn(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                uint32_t blocks) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  ATS_TRY(encode_fn(&enc));
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15) || inner % 64 != 0 || inner == 0 || outer == 0)
    return fail(ATS_EBADARG, "moe_gemm: operand not TMA-compatible (base %p, row %llu B, %llu x %llu)", base,
                (unsigned long long)row_bytes, (unsigned long long)inner, (unsigned long long)outer);
  cuuint64_t dims[3] = {64, outer, inner / 64};
  cuuint64_t strides[2] = {row_bytes, 128};
  cuuint32_t box[3] = {64, 64, blocks};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ATS_ECUDA, "moe_gemm: cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return ATS_OK;
}

// 64-column blocks of an MN-major B tile held by one CTA.
uint32_t b_blocks(int bn, bool pair) { return (pair ? (uint32_t)bn / 2 : (uint32_t)bn) / 64u; }

// Operand map: 128-byte swizzle, box {64, box_outer}.
int make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
             uint32_t box_outer) {
  return encode_map(m, base, inner, outer, row_bytes, 64, box_outer, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Output map of the staged epilogue: 64-byte swizzle, box {32, 32} (one warp's chunk).
int make_out_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes) {
  return encode_map(m, base, inner, outer, row_bytes, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool KGROUP, int SPLIT = 1, int BPARTS = 1, bool PAIR = false>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& p, int64_t max_tiles,
              cudaStream_t st, const CUtensorMap* to = nullptr, const CUtensorMap* to2 = nullptr) {
  auto kfn = tc_gemm_kernel<BN, A_MN, B_MN, EPI, KGROUP, SPLIT, BPARTS, PAIR>;
  if (staging_bytes(EPI) > 0 && to == nullptr) return fail(ATS_EBADARG, "moe_gemm: bf16 epilogue needs an output map");
  if (EPI == EPI_SWIGLU_FWD && to2 == nullptr) return fail(ATS_EBADARG, "moe_gemm: SwiGLU epilogue needs the a map");
  const int smem = 1024 + ring_stages(BN, BPARTS, PAIR, EPI) * stage_bytes(BN, BPARTS, PAIR) + staging_bytes(EPI);
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(ATS_ECUDA, "moe_gemm: smem attribute: %s", cudaGetErrorString(e));
  const CUtensorMap& mo = to != nullptr ? *to : ta;
  const CUtensorMap& mo2 = to2 != nullptr ? *to2 : ta;
  if constexpr (!PAIR) {
    int grid = gemm_ctas();
    if (max_tiles < grid) grid = (int)(max_tiles > 0 ? max_tiles : 1);
    kfn<<<grid, kThreads, smem, st>>>(ta, tb, mo, mo2, p);
  } else {
    // clusters of two CTAs: as many pairs as fit at once on the SMs this GEMM may use
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int pairs = gemm_ctas() / 2;
    static thread_local int fit[kMaxDevices] = {};  // co-resident pairs of this kernel, per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
      return fail(ATS_ECUDA, "moe_gemm: no current device");
    if (fit[dev] == 0) {
      cfg.gridDim = dim3(2 * (unsigned)(pairs > 0 ? pairs : 1), 1, 1);
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kfn, &cfg);
      if (e != cudaSuccess || n < 1) return fail(ATS_ECUDA, "moe_gemm: no CTA pair fits (%s)", cudaGetErrorString(e));
      fit[dev] = n;
    }
    if (pairs > fit[dev]) pairs = fit[dev];
    if (max_tiles < pairs) pairs = (int)(max_tiles > 0 ? max_tiles : 1);
    if (pairs < 1) pairs = 1;
    cfg.gridDim = dim3(2 * (unsigned)pairs, 1, 1);
    e = cudaLaunchKernelEx(&cfg, kfn, ta, tb, mo, mo2, p);
    if (e != cudaSuccess) return fail(ATS_ECUDA, "moe_gemm: pair launch: %s", cudaGetErrorString(e));
  }
  return check_launch("moe_tc_gemm");
}

// The expert GEMMs (one B part, no K parts) on CTA pairs or on single CTAs.  `pair` is read once per entry
// point (gemm_pairs()), so its tensor maps and its launches agree.  A K-major B operand's tensor map has
// boxes of b_box_rows(bn, pair) rows.
template <int BN, bool A_MN, bool B_MN, int EPI, bool KGROUP>
int launch_gemm(bool pair, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& p, int64_t max_tiles,
                cudaStream_t st, const CUtensorMap* to, const CUtensorMap* to2 = nullptr) {
  if (pair) return launch_tc<BN, A_MN, B_MN, EPI, KGROUP, 1, 1, true>(ta, tb, p, max_tiles, st, to, to2);
  return launch_tc<BN, A_MN, B_MN, EPI, KGROUP, 1, 1, false>(ta, tb, p, max_tiles, st, to, to2);
}

uint32_t b_box_rows(int bn, bool pair) { return pair ? (uint32_t)bn / 2 : (uint32_t)bn; }

int pick_bn(int64_t n) { return n % 256 == 0 ? 256 : 128; }

}  // namespace

int tc_experts_fwd(const void* xp, const void* wgu, const void* wd, void* h, void* a, void* y, int E, int64_t H,
                   int64_t F, const SegTable& sg, cudaStream_t st, int64_t io_rows) {
  if (!tc_shape_supported(H, F)) return ATS_EUNSUPPORTED;
  const int64_t R = sg.max_rows;
  const int64_t IO = io_rows > 0 ? io_rows : R;  // rows of xp and y (reads past them are zero, stores clipped)
  const bool pair = gemm_pairs();
  CUtensorMap ma, mb;
  GemmArgs p{};
  p.seg = sg;
  p.F = (int)F;
  // h = xp Wgu_e^T with the SwiGLU epilogue: tile N = 128 gate + 128 up columns
  ATS_TRY(make_map(&ma, xp, H, IO, H * 2, 128));
  ATS_TRY(make_map(&mb, wgu, H, (uint64_t)E * 2 * F, H * 2, 128));
  p.N = (int)F;
  p.K = (int)H;
  p.b = OpSpec{(int)(2 * F), (int)F};
  p.h_out = static_cast<bf16*>(h);
  p.a_out = static_cast<bf16*>(a);
  CUtensorMap mh, mact;
  ATS_TRY(make_out_map(&mh, h, 2 * F, R, 2 * F * 2));
  ATS_TRY(make_out_map(&mact, a, F, R, F * 2));
  ATS_TRY((launch_gemm<256, false, false, EPI_SWIGLU_FWD, false>(pair, ma, mb, p, (R / BM) * (F / 128), st, &mh,
                                                                  &mact)));
  // y = a Wd_e^T
  const int bn = pick_bn(H);
  ATS_TRY(make_map(&ma, a, F, R, F * 2, 128));
  ATS_TRY(make_map(&mb, wd, F, (uint64_t)E * H, F * 2, b_box_rows(bn, pair)));
  p.N = (int)H;
  p.K = (int)F;
  p.b = OpSpec{(int)H, 0};
  p.out = static_cast<bf16*>(y);
  p.ldo = H;
  CUtensorMap mo;
  ATS_TRY(make_out_map(&mo, y, H, IO, H * 2));
  if (bn == 256) return launch_gemm<256, false, false, EPI_STORE, false>(pair, ma, mb, p, (R / BM) * (H / 256), st, &mo);
  return launch_gemm<128, false, false, EPI_STORE, false>(pair, ma, mb, p, (R / BM) * (H / 128), st, &mo);
}

int tc_experts_bwd(const void* dy, const void* xp, const void* h, const void* a, const void* wgu, const void* wd,
                   void* dh, void* dxp, void* dwgu, void* dwd, int E, int64_t H, int64_t F, const SegTable& sg,
                   cudaStream_t st, int64_t io_rows, int stages) {
  if (!tc_shape_supported(H, F)) return ATS_EUNSUPPORTED;
  const int64_t R = sg.max_rows;
  const int64_t IO = io_rows > 0 ? io_rows : R;  // rows of dy, xp and dxp
  const bool pair = gemm_pairs();
  CUtensorMap ma, mb;
  GemmArgs p{};
  p.seg = sg;
  p.F = (int)F;
  // da = dy Wd_e (B N-major: Wd_e[h][f]) with the SwiGLU backward epilogue -> dh
  if (stages & kBwdData) {
    const int bn = pick_bn(F);
    ATS_TRY(make_map(&ma, dy, H, IO, H * 2, 128));
    ATS_TRY(make_map_mn(&mb, wd, F, (uint64_t)E * H, F * 2, b_blocks(bn, pair)));
    p.N = (int)F;
    p.K = (int)H;
    p.b = OpSpec{(int)H, 0};
    p.h = static_cast<const bf16*>(h);
    p.out = static_cast<bf16*>(dh);
    CUtensorMap mdh;
    ATS_TRY(make_out_map(&mdh, dh, 2 * F, R, 2 * F * 2));
    if (bn == 256)
      ATS_TRY((launch_gemm<256, false, true, EPI_SWIGLU_BWD, false>(pair, ma, mb, p, (R / BM) * (F / 256), st, &mdh)));
    else
      ATS_TRY((launch_gemm<128, false, true, EPI_SWIGLU_BWD, false>(pair, ma, mb, p, (R / BM) * (F / 128), st, &mdh)));
  }
  // dxp = dh Wgu_e (B N-major: Wgu_e[j][h])
  if (stages & kBwdData) {
    const int bn = pick_bn(H);
    ATS_TRY(make_map(&ma, dh, 2 * F, R, 2 * F * 2, 128));
    ATS_TRY(make_map_mn(&mb, wgu, H, (uint64_t)E * 2 * F, H * 2, b_blocks(bn, pair)));
    p.N = (int)H;
    p.K = (int)(2 * F);
    p.b = OpSpec{(int)(2 * F), 0};
    p.out = static_cast<bf16*>(dxp);
    p.ldo = H;
    CUtensorMap mo;
    ATS_TRY(make_out_map(&mo, dxp, H, IO, H * 2));
    if (bn == 256)
      ATS_TRY((launch_gemm<256, false, true, EPI_STORE, false>(pair, ma, mb, p, (R / BM) * (H / 256), st, &mo)));
    else
      ATS_TRY((launch_gemm<128, false, true, EPI_STORE, false>(pair, ma, mb, p, (R / BM) * (H / 128), st, &mo)));
  }
  if (!(stages & kBwdWeights)) return ATS_OK;
  // dWd_e[h][f] = sum over the expert's rows r of dy[r][h] a[r][f]   (A M-major, B N-major).  256-wide tiles
  // even when F is an odd multiple of 128: the last tile's upper half reads zeros and stores nothing, and the
  // wider tiles read each row's operands half as often (these GEMMs have a short K: an expert's rows)
  {
    const int bn = 256;
    ATS_TRY(make_map_mn(&ma, dy, H, IO, H * 2, 2));
    ATS_TRY(make_map_mn(&mb, a, F, R, F * 2, b_blocks(bn, pair)));
    p.M = (int)H;
    p.N = (int)F;
    p.K = 0;
    p.b = OpSpec{0, 0};
    p.out = static_cast<bf16*>(dwd);
    p.ldo = F;
    p.out_group = H * F;
    CUtensorMap mo;
    ATS_TRY(make_out_map(&mo, dwd, F, (uint64_t)sg.E * H, F * 2));
    const int64_t tiles = (int64_t)sg.E * (H / BM) * ((F + bn - 1) / bn);
    ATS_TRY((launch_gemm<256, true, true, EPI_STORE, true>(pair, ma, mb, p, tiles, st, &mo)));
  }
  // dWgu_e[j][h] = sum over the expert's rows r of dh[r][j] xp[r][h]
  {
    const int bn = pick_bn(H);
    ATS_TRY(make_map_mn(&ma, dh, 2 * F, R, 2 * F * 2, 2));
    ATS_TRY(make_map_mn(&mb, xp, H, IO, H * 2, b_blocks(bn, pair)));
    p.M = (int)(2 * F);
    p.N = (int)H;
    p.out = static_cast<bf16*>(dwgu);
    p.ldo = H;
    p.out_group = 2 * F * H;
    CUtensorMap mo;
    ATS_TRY(make_out_map(&mo, dwgu, H, (uint64_t)sg.E * 2 * F, H * 2));
    const int64_t tiles = (int64_t)sg.E * (2 * F / BM) * (H / bn);
    if (bn == 256) return launch_gemm<256, true, true, EPI_STORE, true>(pair, ma, mb, p, tiles, st, &mo);
    return launch_gemm<128, true, true, EPI_STORE, true>(pair, ma, mb, p, tiles, st, &mo);
  }
}



// C[M,N] = A[M,K] B[N,K]^T with the rotary embedding applied to each 128-column head of C in the epilogue
// (the q/k projection of attention followed by apply_rotary_pos_emb).  C has row stride ldc elements.
int tc_gemm_rope_fwd(const void* a, const void* b, void* c, int64_t ldc, int64_t N, int64_t K, const void* cos,
                     const void* sin, int64_t seq, const SegTable& sg, cudaStream_t st, int64_t io_rows) {
  if (!tc_shape_supported(N, K)) return ATS_EUNSUPPORTED;
  const int64_t R = sg.max_rows;
  CUtensorMap ma, mb, mo;
  GemmArgs p{};
  p.seg = sg;
  ATS_TRY(make_map(&ma, a, K, io_rows, K * 2, 128));
  ATS_TRY(make_map(&mb, b, K, N, K * 2, 128));
  p.N = (int)N;
  p.K = (int)K;
  p.b = OpSpec{(int)N, 0};
  p.out = static_cast<bf16*>(c);
  p.ldo = ldc;
  p.m_valid = (int)io_rows;
  p.rope_cos = static_cast<const bf16*>(cos);
  p.rope_sin = static_cast<const bf16*>(sin);
  p.rope_seq = (int)seq;
  ATS_TRY(make_out_map(&mo, c, N, io_rows, ldc * 2));
  return launch_tc<128, false, false, EPI_ROPE, false>(ma, mb, p, (R / BM) * (N / 128), st, &mo);
}

// Plain GEMM on the same kernel, one segment over the rows (the dense table):
// C[M,N] = A[M,K] B[N,K]^T.  A and C have io_rows rows (reads past them are zero,
// stores clipped); the tiles cover sg.max_rows = M rounded up to 128.
int tc_gemm_nt_fwd(const void* a, const void* b, void* c, int64_t N, int64_t K, const SegTable& sg, cudaStream_t st,
                   int64_t io_rows) {
  if (!tc_shape_supported(N, K)) return ATS_EUNSUPPORTED;
  const int64_t R = sg.max_rows;
  const int bn = pick_bn(N);
  const bool pair = gemm_pairs();
  CUtensorMap ma, mb, mo;
  GemmArgs p{};
  p.seg = sg;
  ATS_TRY(make_map(&ma, a, K, io_rows, K * 2, 128));
  ATS_TRY(make_map(&mb, b, K, N, K * 2, b_box_rows(bn, pair)));
  p.N = (int)N;
  p.K = (int)K;
  p.b = OpSpec{(int)N, 0};
  p.out = static_cast<bf16*>(c);
  p.ldo = N;
  ATS_TRY(make_out_map(&mo, c, N, io_rows, N * 2));
  if (bn == 256) return launch_gemm<256, false, false, EPI_STORE, false>(pair, ma, mb, p, (R / BM) * (N / 256), st, &mo);
  return launch_gemm<128, false, false, EPI_STORE, false>(pair, ma, mb, p, (R / BM) * (N / 128), st, &mo);
}

// Its gradients: dA[M,K] = dC[M,N] B[N,K] (B N-major), dB[N,K] = dC^T A summed over the
// rows (K-grouped, both operands MN-major).  A null da or db skips that GEMM.
int tc_gemm_nt_bwd(const void* dc, const void* a, const void* b, void* da, void* db, int64_t N, int64_t K,
                   const SegTable& sg, cudaStream_t st, int64_t io_rows) {
  if (!tc_shape_supported(N, K)) return ATS_EUNSUPPORTED;
  const int64_t R = sg.max_rows;
  const bool pair = gemm_pairs();
  if (da != nullptr) {
    const int bn = pick_bn(K);
    CUtensorMap ma, mb, mo;
    GemmArgs p{};
    p.seg = sg;
    ATS_TRY(make_map(&ma, dc, N, io_rows, N * 2, 128));
    ATS_TRY(make_map_mn(&mb, b, K, N, K * 2, b_blocks(bn, pair)));
    p.N = (int)K;
    p.K = (int)N;
    p.b = OpSpec{(int)N, 0};
    p.out = static_cast<bf16*>(da);
    p.ldo = K;
    ATS_TRY(make_out_map(&mo, da, K, io_rows, K * 2));
    if (bn == 256)
      ATS_TRY((launch_gemm<256, false, true, EPI_STORE, false>(pair, ma, mb, p, (R / BM) * (K / 256), st, &mo)));
    else
      ATS_TRY((launch_gemm<128, false, true, EPI_STORE, false>(pair, ma, mb, p, (R / BM) * (K / 128), st, &mo)));
  }
  if (db != nullptr) {
    const int bn = pick_bn(K);
    CUtensorMap ma, mb, mo;
    GemmArgs p{};
    p.seg = sg;
    ATS_TRY(make_map_mn(&ma, dc, N, io_rows, N * 2, 2));
    ATS_TRY(make_map_mn(&mb, a, K, io_rows, K * 2, b_blocks(bn, pair)));
    p.M = (int)N;
    p.N = (int)K;
    p.K = 0;
    p.b = OpSpec{0, 0};
    p.out = static_cast<bf16*>(db);
    p.ldo = K;
    p.out_group = N * K;
    ATS_TRY(make_out_map(&mo, db, K, N, K * 2));
    const int64_t tiles = (N / BM) * (K / bn);
    if (bn == 256) return launch_gemm<256, true, true, EPI_STORE, true>(pair, ma, mb, p, tiles, st, &mo);
    return launch_gemm<128, true, true, EPI_STORE, true>(pair, ma, mb, p, tiles, st, &mo);
  }
  return ATS_OK;
}

namespace {
void set_parts(int (&dst)[kMaxParts], std::initializer_list<int> v) {
  int i = 0;
  for (int x : v) dst[i++] = x;
  for (; i < kMaxParts; ++i) dst[i] = 0;
}
}  // namespace

int tc_router_logits(const void* x, const void* wparts, const float* bias, float* logits, int64_t T, int64_t H,
                     int E, int Ep, const SegTable& one, cudaStream_t st) {
  if (Ep != kRouterEp) return fail(ATS_EUNSUPPORTED, "moe_router: padded expert count %d", Ep);
  CUtensorMap ma, mb;
  GemmArgs p{};
  p.seg = one;
  p.N = Ep;
  p.K = (int)H;
  p.b = OpSpec{0, 0};
  set_parts(p.b_noff, {0, Ep, 2 * Ep});  // the three weight parts, consecutive rows: one box per k block
  p.out_f32 = logits;
  p.ldo = E;
  p.bias = bias;
  p.m_valid = (int)T;
  p.n_valid = E;
  ATS_TRY(make_map(&ma, x, H, T, H * 2, 128));
  ATS_TRY(make_map(&mb, wparts, H, (uint64_t)3 * Ep, H * 2, 3 * Ep));
  return launch_tc<kRouterEp, false, false, EPI_F32, false, 1, 3>(ma, mb, p, (T + BM - 1) / BM, st);
}

int tc_router_dx(const void* dlparts, const void* wparts, const void* dxp, const int* tok_row, int k, void* dx,
                 int64_t T, int64_t H, int Ep, const SegTable& one, cudaStream_t st) {
  CUtensorMap ma, mb;
  GemmArgs p{};
  p.seg = one;
  p.N = (int)H;
  p.K = Ep;
  p.b = OpSpec{0, 0};
  // dl . w over the six part pairs whose product is above 2^-24 of the leading one
  set_parts(p.a_koff, {0, 0, 0, Ep, Ep, 2 * Ep});
  set_parts(p.b_koff, {0, Ep, 2 * Ep, 0, Ep, 0});
  set_parts(p.b_noff, {0, 0, 0, 0, 0, 0});
  p.out = static_cast<bf16*>(dx);
  p.ldo = H;
  p.m_valid = (int)T;
  p.n_valid = (int)H;
  p.dxp = static_cast<const bf16*>(dxp);
  p.tok_row = tok_row;
  p.topk = k;
  ATS_TRY(make_map(&ma, dlparts, (uint64_t)3 * Ep, T, (uint64_t)3 * Ep * 2, 128));
  if (Ep != kRouterEp) return fail(ATS_EUNSUPPORTED, "moe_router: padded expert count %d", Ep);
  ATS_TRY(make_map_mn(&mb, wparts, H, (uint64_t)3 * Ep, H * 2, b_blocks(pick_bn(H), false)));
  CUtensorMap mo;
  ATS_TRY(make_out_map(&mo, dx, H, T, H * 2));
  const int64_t mt = (T + BM - 1) / BM;
  if (pick_bn(H) == 256)
    return launch_tc<256, false, true, EPI_SCATTER, false, 6>(ma, mb, p, mt * (H / 256), st, &mo);
  return launch_tc<128, false, true, EPI_SCATTER, false, 6>(ma, mb, p, mt * (H / 128), st, &mo);
}

int tc_router_dw(const void* x, const void* dlparts, float* partial, int64_t T, int64_t H, int Ep,
                 const SegTable& chunks, cudaStream_t st) {
  if (Ep != kRouterEp) return fail(ATS_EUNSUPPORTED, "moe_router: padded expert count %d", Ep);
  CUtensorMap ma, mb;
  GemmArgs p{};
  p.seg = chunks;
  p.M = (int)H;
  p.N = Ep;
  p.K = 0;
  p.b = OpSpec{0, 0};
  set_parts(p.b_noff, {0, Ep, 2 * Ep});  // the three gradient parts, consecutive columns: one load per k block
  p.out_f32 = partial;
  p.ldo = Ep;
  p.out_group = H * Ep;
  p.m_valid = (int)H;
  p.n_valid = Ep;
  ATS_TRY(make_map_mn(&ma, x, H, T, H * 2, 2));
  ATS_TRY(make_map_mn(&mb, dlparts, (uint64_t)3 * Ep, T, (uint64_t)3 * Ep * 2, 3));
  return launch_tc<kRouterEp, true, true, EPI_F32, true, 1, 3>(ma, mb, p, (int64_t)chunks.E * (H / BM), st);
}

int gemm_set_wait_budget(long long cycles) {
  const long long v = cycles > 0 ? cycles : kWaitBudget;
  cudaError_t e = cudaMemcpyToSymbol(g_gemm_wait_budget, &v, sizeof(v));
  if (e != cudaSuccess) return fail(ATS_ECUDA, "set_wait_budget (gemm): %s", cudaGetErrorString(e));
  return ATS_OK;
}

int gemm_take_status(int* code) {
  const int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(code, g_gemm_status, sizeof(int));
  if (e == cudaSuccess && *code != 0) e = cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int));
  if (e != cudaSuccess) return fail(ATS_ECUDA, "device_status (gemm): %s", cudaGetErrorString(e));
  return ATS_OK;
}

}  // namespace ats
