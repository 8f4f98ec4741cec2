// N7 / N8: grouped expert GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   GROUP_M:  C[off_e : off_e+m_e, :] = A[off_e : off_e+m_e, :] @ B[e]^T      (forward, dX)
//   GROUP_K:  C[e] = A[:, off_e : off_e+m_e] @ B[:, off_e : off_e+m_e]^T          (dW)
//
// A, B are bf16, each either K-major (the reduction dimension is contiguous) or
// MN-major (the output dimension is contiguous), so transposed operands are read
// in place instead of being materialised: the backward's dX GEMM takes the
// forward weight [G, K, N] as an MN-major B, and the weight-gradient GEMM takes
// the activations [tokens, M] and [tokens, N] as MN-major A and B. Expert
// segments are padded to multiples of 128 rows (the permute kernel does this),
// so every M tile (GROUP_M) or K block (GROUP_K) lies inside one expert.
//
// Per CTA (one per SM, persistent over tiles), 6 warps:
//   warp 0      TMA producer: one elected thread streams A/B k-blocks (128B-swizzled
//               boxes, each CTA loading its own) into a STAGES-deep shared-memory ring.
//   warp 1      TMEM owner + MMA issuer: allocates 512 TMEM columns (two 128x256
//               fp32 accumulators), one elected thread issues tcgen05.mma
//               (M=128, N=BN, K=16) per 16-wide k slice and commits each stage
//               back to the producer and each finished tile to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (thread = row), fused
//               activation (SwiGLU on interleaved gate/up blocks) and the bf16/fp32
//               cast into a swizzled 32x32 box in shared memory, which one lane
//               stores with a TMA tensor store (the map clips rows and columns past
//               the output's extent); the accumulator is freed as soon as it has
//               been read, so the stores overlap the next tile's MMAs.
// Every mbarrier wait is bounded; on timeout the CTA records an error, stops
// issuing, frees its TMEM and returns.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "ops.h"

namespace b200ep {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;           // 64 bf16 = 128 bytes = one swizzle row
constexpr int UMMA_K = 16;
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;

enum Epilogue : int { kEpiBF16 = 0, kEpiF32 = 1, kEpiSwiGLU = 2 };

struct Args {
  const int64_t* offsets;   // [G + 1] row (GROUP_M) or token (GROUP_K) offsets, multiples of 128
  int G;
  int M, N, K;              // GROUP_M: N, K fixed, M = rows of A (bounds the offsets). GROUP_K: M, N fixed.
  void* C;
  int64_t ldc;              // elements
  void* H;                  // SwiGLU output [rows, N/2] bf16
  int64_t ldh;
  int64_t c_group_stride;   // GROUP_K: elements between experts' outputs
  int64_t c_rows;           // GROUP_M: rows of C (and H); later tile rows are not stored
  const void* R;            // GROUP_M bf16 epilogue: optional residual [rows, N] added before rounding
  int64_t ldr;
  uint32_t* error;          // device word, non-zero after a timeout
  uint64_t timeout_ns;
  // fp8 block-scaled mode: scales as 512-byte tiles, one per (128 rows, 128-channel K block),
  // already in the layout tcgen05.cp moves to tensor memory (see sf_tiles_kernel)
  const uint8_t* sfa_tiles; // [ceil(rows / 128), K / 128, 512 B]
  const uint8_t* sfb_tiles; // [G, ceil(N / 128), K / 128, 512 B]
};

// ----------------------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void tma_load_2d(void* smem, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// shared -> global tensor stores (bulk async-group of the calling thread)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(smem)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(smem_u32(smem)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D (+)= (A * SFA) x (B * SFB)^T for e4m3 operands, K = 32 per instruction, with one UE8M0
// scale per 32 K-elements of each row of A and of B read from tensor memory.
__device__ __forceinline__ void tc_mma_fp8_bs(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate, uint32_t tmem_sfa, uint32_t tmem_sfb) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tmem_sfa), "r"(tmem_sfb)
      : "memory");
}
// 32 rows x 16 bytes of shared memory -> 32 TMEM lanes x 4 columns, written to all four
// 32-lane subpartitions (the replicated layout the block-scaled MMA reads scales from).
__device__ __forceinline__ void tc_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets row (lane base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 bytes,
// 8-row groups 1024 bytes apart (the layout a SWIZZLE_128B TMA box produces).
__device__ __forceinline__ uint64_t smem_desc_k128(const void* p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = (addr >> 4) & 0x3FFFull;   // start address
  d |= 1ull << 16;                         // leading byte offset (unused for swizzled K-major)
  d |= (1024ull >> 4) << 32;               // stride byte offset: 8 rows x 128 B
  d |= 1ull << 46;                         // descriptor version for sm_100
  d |= 2ull << 61;                         // SWIZZLE_128B
  return d;
}
// MN-major, 128-byte swizzle: each 128-byte row holds 64 consecutive M (or N) elements
// of one k, 8 k-rows form a 1024-byte swizzle atom (stride byte offset), and the
// 64-wide MN atoms of a tile sit `mn_atom_bytes` apart (leading byte offset). This is
// what a SWIZZLE_128B TMA box of 64 (MN) x BK (K) elements produces, one box per atom.
__device__ __forceinline__ uint64_t smem_desc_mn128(const void* p, uint32_t mn_atom_bytes) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = (addr >> 4) & 0x3FFFull;
  d |= static_cast<uint64_t>((mn_atom_bytes >> 4) & 0x3FFFu) << 16;
  d |= (1024ull >> 4) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}
// Instruction descriptor: D fp32, A/B bf16, M=128, N=n; bits 15 / 16 select MN-major A / B.
__host__ __device__ constexpr uint32_t idesc_bf16(int n, bool a_mn = false, bool b_mn = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}
constexpr uint32_t kMnAtomBytes = 64 * BK * 2;  // one 64-wide MN column of a BK-deep stage

// Instruction descriptor of the block-scaled fp8 MMA: A/B e4m3, K-major, UE8M0 scales,
// scale byte 0 of each TMEM word for both operands, M=128, N=n, K=32.
__host__ __device__ constexpr uint32_t idesc_fp8_bs(int n) {
  return (0u << 4) | (0u << 7) | (0u << 10) | (uint32_t(n >> 3) << 17) | (1u << 23) | (uint32_t(BM >> 4) << 24);
}
// Shared-memory descriptor of a dense, unswizzled 32-row x 16-byte tile (the source of
// tcgen05.cp 32x128b): rows 16 bytes apart, 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sf(const void* p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = (addr >> 4) & 0x3FFFull;
  d |= (128ull >> 4) << 16;   // leading byte offset (a single core matrix along K: unused)
  d |= (128ull >> 4) << 32;   // stride byte offset: next 8 rows
  d |= 1ull << 46;            // descriptor version for sm_100; layout type 0 = no swizzle
  return d;
}
// fp8 mode: K elements per pipeline stage (128 one-byte elements fill the 128-byte swizzle row)
constexpr int BK8 = 128;
// Scale-factor staging per stage: SFA (128 rows) then SFB (BN rows), 16 bytes per 4 rows.
template <int BN>
__host__ __device__ constexpr int sf_stage_bytes() { return (BM + BN) * 4; }

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, const Args& a) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > a.timeout_ns || *reinterpret_cast<volatile uint32_t*>(a.error) != 0u) {
      atomicExch(a.error, 1u);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ float silu(float g) { return g / (1.f + __expf(-g)); }

template <int BN>
struct Smem {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
};
// Epilogue staging: per epilogue warp, a ring of 32 x 32 output boxes (2 KB bf16 with
// 64-byte rows and SWIZZLE_64B, or 4 KB fp32 with 128-byte rows and SWIZZLE_128B).
constexpr int kEpiWarpBytes = 4096;
constexpr int kEpiBytes = 4 * kEpiWarpBytes;

// Row r (= lane) of a 32 x 32 box into its swizzled slot: 16-byte chunk c of the row
// goes to chunk c ^ (swizzle phase of row r), the pattern the tensor map's swizzle mode
// undoes on the way out; the 8 rows of each 128-byte bank window land in distinct banks.
__device__ __forceinline__ void put_row_bf16(uint8_t* slot, int r, const uint32_t (&v)[16]) {
  const int4* src = reinterpret_cast<const int4*>(v);
#pragma unroll
  for (int c = 0; c < 4; ++c) *reinterpret_cast<int4*>(slot + r * 64 + ((c ^ ((r >> 1) & 3)) << 4)) = src[c];
}
__device__ __forceinline__ void put_row_f32(uint8_t* slot, int r, const uint32_t (&v)[32]) {
  const int4* src = reinterpret_cast<const int4*>(v);
#pragma unroll
  for (int c = 0; c < 8; ++c) *reinterpret_cast<int4*>(slot + r * 128 + ((c ^ (r & 7)) << 4)) = src[c];
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

// Tile t -> (group, m0 / k range, n0). Returns false past the end.
struct Tile {
  int g;
  int m0, n0;
  int kb0, nkb;  // k-block range
};

template <bool GROUP_K, int BN, int KBLK = BK>
__device__ __forceinline__ bool tile_of(int t, const Args& a, const int64_t* offs, Tile& tl) {
  const int ntiles_n = (a.N + BN - 1) / BN;
  if (!GROUP_K) {
    // tiles cover min(offsets[G], rows of A rounded up); rows past C are masked in the epilogue
    const int64_t mpad = (static_cast<int64_t>(a.M) + BM - 1) / BM * BM;
    const int total_m = static_cast<int>((offs[a.G] < mpad ? offs[a.G] : mpad) / BM);
    if (t >= total_m * ntiles_n) return false;
    const int mt = t / ntiles_n;
    tl.n0 = (t % ntiles_n) * BN;
    tl.m0 = mt * BM;
    int lo = 0, hi = a.G - 1;  // last group with offs[g] <= m0
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (offs[mid] <= tl.m0) lo = mid; else hi = mid - 1;
    }
    tl.g = lo;
    tl.kb0 = 0;
    tl.nkb = (a.K + KBLK - 1) / KBLK;
  } else {
    const int ntiles_m = (a.M + BM - 1) / BM;
    const int per = ntiles_m * ntiles_n;
    if (t >= per * a.G) return false;
    tl.g = t / per;
    const int r = t % per;
    tl.m0 = (r / ntiles_n) * BM;
    tl.n0 = (r % ntiles_n) * BN;
    tl.kb0 = static_cast<int>(offs[tl.g] / BK);
    tl.nkb = static_cast<int>((offs[tl.g + 1] - offs[tl.g]) / BK);
  }
  return true;
}

// LAYOUT bit 0: A is MN-major; bit 1: B is MN-major (GROUP_M: B is [G, K, N], read
// through a 3-D map so a K tail never reaches into the next expert's weight).
// FP8: A and B are e4m3 (K-major, GROUP_M only) with power-of-two fp32 scales per
// (row, 128-channel block); the MMA applies them (kind::mxf8f6f4.block_scale).
template <bool GROUP_K, int BN, int STAGES, int EPI, int LAYOUT, bool FP8 = false>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmH, Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  using S = Smem<BN>;
  constexpr bool A_MN = (LAYOUT & 1) != 0, B_MN = (LAYOUT & 2) != 0;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kABytes;
  uint8_t* sE = sB + STAGES * S::kBBytes;  // epilogue staging, kEpiWarpBytes per epilogue warp
  uint8_t* sSF = sE + kEpiBytes;           // fp8 mode: per-stage scale tiles
  constexpr int kSF = FP8 ? sf_stage_bytes<BN>() : 0;
  constexpr int KBLK = FP8 ? BK8 : BK;     // K elements per stage
  static_assert(!FP8 || (!GROUP_K && LAYOUT == 0 && BN <= 128), "fp8: grouped-M, K-major, N tile <= 128");
  uint64_t* full = reinterpret_cast<uint64_t*>(sSF + STAGES * kSF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int64_t s_offs[1025];
  __shared__ volatile int s_abort;

  const int warp = warp_id(), lane = lane_id();
  for (int i = threadIdx.x; i <= a.G && i <= 1024; i += kThreads) s_offs[i] = a.offsets[i];
  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
    if (EPI == kEpiSwiGLU) prefetch_tmap(&tmH);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (FP8 && warp == 0) {
    // ------------------------------------------------------------------ TMA producer (fp8)
    // per stage: the A and B tiles plus their two 512-byte scale tiles (bulk copies)
    if (lane == 0) {
      uint32_t it = 0;
      Tile tl;
      const int KB = (a.K + KBLK - 1) / KBLK;
      const int ntn = (a.N + BN - 1) / BN;
      for (int t = blockIdx.x; tile_of<GROUP_K, BN, KBLK>(t, a, s_offs, tl) && !s_abort; t += gridDim.x) {
        for (int kb = 0; kb < tl.nkb; ++kb, ++it) {
          const int s = it % STAGES;
          if (!wait_bar(&empty[s], ((it / STAGES) & 1u) ^ 1u, a)) { s_abort = 1; break; }
          mbar_arrive_expect_tx(&full[s], S::kStageBytes + kSF);
          const int kg = tl.kb0 + kb;
          const int kc = kg * KBLK;
          tma_load_2d(sA + s * S::kABytes, &tmA, &full[s], kc, tl.m0);
          tma_load_2d(sB + s * S::kBBytes, &tmB, &full[s], kc, tl.g * a.N + tl.n0);
          uint8_t* sf = sSF + s * kSF;
          bulk_load(sf, a.sfa_tiles + (static_cast<int64_t>(tl.m0 / BM) * KB + kg) * 512, 512, &full[s]);
          bulk_load(sf + 512,
                    a.sfb_tiles + ((static_cast<int64_t>(tl.g) * ntn + tl.n0 / BN) * KB + kg) * 512, 512, &full[s]);
        }
      }
    }
  } else if (!FP8 && warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      Tile tl;
      for (int t = blockIdx.x; tile_of<GROUP_K, BN>(t, a, s_offs, tl) && !s_abort; t += gridDim.x) {
        for (int kb = 0; kb < tl.nkb; ++kb, ++it) {
          const int s = it % STAGES;
          if (!wait_bar(&empty[s], ((it / STAGES) & 1u) ^ 1u, a)) { s_abort = 1; break; }
          mbar_arrive_expect_tx(&full[s], S::kStageBytes);
          const int kc = (tl.kb0 + kb) * BK;
          uint8_t* da = sA + s * S::kABytes;
          uint8_t* db = sB + s * S::kBBytes;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(da + j * kMnAtomBytes, &tmA, &full[s], tl.m0 + 64 * j, kc);
          } else {
            tma_load_2d(da, &tmA, &full[s], kc, tl.m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              if (!GROUP_K) tma_load_3d(db + j * kMnAtomBytes, &tmB, &full[s], tl.n0 + 64 * j, kc, tl.g);
              else tma_load_2d(db + j * kMnAtomBytes, &tmB, &full[s], tl.n0 + 64 * j, kc);
            }
          } else {
            tma_load_2d(db, &tmB, &full[s], kc, GROUP_K ? tl.n0 : tl.g * a.N + tl.n0);
          }
        }
      }
    }
  } else if (FP8 && warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (fp8, block-scaled)
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_fp8_bs(BN);
      constexpr uint32_t kSfCol0 = 2 * BN;   // scale columns follow the two accumulators
      uint32_t it = 0, acc = 0;
      Tile tl;
      for (int t = blockIdx.x; tile_of<GROUP_K, BN, KBLK>(t, a, s_offs, tl) && !s_abort; t += gridDim.x) {
        if (tl.nkb == 0) continue;
        const int b = acc & 1;
        if (!wait_bar(&tempty[b], ((acc >> 1) & 1u) ^ 1u, a)) { s_abort = 1; break; }
        tc_fence_after();
        const uint32_t dcol = tmem_base + b * BN;
        bool ok = true;
        for (int kb = 0; kb < tl.nkb; ++kb, ++it) {
          const int s = it % STAGES;
          if (!wait_bar(&full[s], (it / STAGES) & 1u, a)) { ok = false; break; }
          tc_fence_after();
          // this stage's scales: SFA in 4 columns, SFB in BN / 32 columns
          const uint32_t sfa_t = tmem_base + kSfCol0 + s * (4 + BN / 32);
          const uint32_t sfb_t = sfa_t + 4;
          const uint8_t* sf = sSF + s * kSF;
          tc_cp_32x128b_x4(sfa_t, smem_desc_sf(sf));
#pragma unroll
          for (int j = 0; j < BN / 128; ++j) tc_cp_32x128b_x4(sfb_t + 4 * j, smem_desc_sf(sf + 512 + 512 * j));
          const uint64_t ad = smem_desc_k128(sA + s * S::kABytes);
          const uint64_t bd = smem_desc_k128(sB + s * S::kBBytes);
          // 4 MMAs of K = 32 one-byte elements: 32 bytes (2 units) along the swizzle row each
#pragma unroll
          for (int k = 0; k < BK8 / 32; ++k)
            tc_mma_fp8_bs(dcol, ad + 2 * k, bd + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u, sfa_t, sfb_t);
          tc_commit(&empty[s]);
        }
        if (!ok) { s_abort = 1; break; }
        tc_commit(&tfull[b]);
        ++acc;
      }
      tc_commit(drain);
      wait_bar(drain, 0, a);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BN, A_MN, B_MN);
      uint32_t it = 0, acc = 0;
      Tile tl;
      for (int t = blockIdx.x; tile_of<GROUP_K, BN>(t, a, s_offs, tl) && !s_abort; t += gridDim.x) {
        if (tl.nkb == 0) continue;  // empty expert: the epilogue writes zeros without the accumulator
        const int b = acc & 1;
        if (!wait_bar(&tempty[b], ((acc >> 1) & 1u) ^ 1u, a)) { s_abort = 1; break; }
        tc_fence_after();
        const uint32_t dcol = tmem_base + b * BN;
        bool ok = true;
        for (int kb = 0; kb < tl.nkb; ++kb, ++it) {
          const int s = it % STAGES;
          if (!wait_bar(&full[s], (it / STAGES) & 1u, a)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = A_MN ? smem_desc_mn128(sA + s * S::kABytes, kMnAtomBytes)
                                   : smem_desc_k128(sA + s * S::kABytes);
          const uint64_t bd = B_MN ? smem_desc_mn128(sB + s * S::kBBytes, kMnAtomBytes)
                                   : smem_desc_k128(sB + s * S::kBBytes);
          // next 16-wide k slice: K-major advances 32 bytes inside the swizzle row (2 units),
          // MN-major advances 16 rows of 128 bytes (128 units)
          constexpr uint64_t astep = A_MN ? 128 : 2, bstep = B_MN ? 128 : 2;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k)
            tc_mma(dcol, ad + astep * k, bd + bstep * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        if (!ok) { s_abort = 1; break; }
        tc_commit(&tfull[b]);
        ++acc;
      }
      // every issued MMA has completed before TMEM is released
      tc_commit(drain);
      wait_bar(drain, 0, a);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;                    // TMEM lane quarter this warp may access
    uint8_t* ring = sE + (warp - 2) * kEpiWarpBytes;
    constexpr int kSlot = EPI == kEpiF32 ? 4096 : 2048;
    constexpr int kSlots = kEpiWarpBytes / kSlot;
    uint32_t nst = 0;                          // boxes this warp has stored (ring position)
    // one 32 x 32 box: wait until its slot's previous store has read it, fill, store
    auto store_box = [&](const CUtensorMap* map, auto&& fill, int x, int y, int g) {
      uint8_t* slot = ring + (nst % kSlots) * kSlot;
      if (lane == 0) bulk_wait_read<kSlots - 1>();
      __syncwarp();
      fill(slot);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (GROUP_K) tma_store_3d(map, slot, x, y, g);
        else tma_store_2d(map, slot, x, y);
        bulk_commit();
      }
      ++nst;
    };
    uint32_t acc = 0;
    Tile tl;
    for (int t = blockIdx.x; tile_of<GROUP_K, BN, KBLK>(t, a, s_offs, tl); t += gridDim.x) {
      const int b = acc & 1;
      const bool have = tl.nkb > 0;
      if (have) {
        if (!wait_bar(&tfull[b], (acc >> 1) & 1u, a)) { s_abort = 1; }
        if (s_abort) break;
        tc_fence_after();
      }
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * BN;
      const int row0 = tl.m0 + q * 32;         // first row of this warp's boxes
      // boxes that start past the output are skipped; the map clips partial ones
      const bool rows_in = GROUP_K ? row0 < a.M : row0 < a.c_rows;
      if (EPI == kEpiSwiGLU) {
        // tile = [128 gate columns | 128 up columns] of the interleaved weight layout
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(taddr + c, g);
          tmem_ld32(taddr + BN / 2 + c, u);
          if (!rows_in) continue;
          uint32_t hv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float g0 = __uint_as_float(g[2 * i]), g1 = __uint_as_float(g[2 * i + 1]);
            const float u0 = __uint_as_float(u[2 * i]), u1 = __uint_as_float(u[2 * i + 1]);
            hv[i] = pack_bf16(silu(g0) * u0, silu(g1) * u1);
          }
          store_box(&tmH, [&](uint8_t* sl) { put_row_bf16(sl, lane, hv); }, tl.n0 / 2 + c, row0, 0);
          if (a.C) {
            uint32_t pv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) pv[i] = pack_bf16(__uint_as_float(g[2 * i]), __uint_as_float(g[2 * i + 1]));
            store_box(&tmC, [&](uint8_t* sl) { put_row_bf16(sl, lane, pv); }, tl.n0 + c, row0, 0);
#pragma unroll
            for (int i = 0; i < 16; ++i) pv[i] = pack_bf16(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1]));
            store_box(&tmC, [&](uint8_t* sl) { put_row_bf16(sl, lane, pv); }, tl.n0 + BN / 2 + c, row0, 0);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          if (have) {
            tmem_ld32(taddr + c, r);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = 0u;
          }
          if (!rows_in || tl.n0 + c >= a.N) continue;
          if (EPI == kEpiF32) {
            store_box(&tmC, [&](uint8_t* sl) { put_row_f32(sl, lane, r); }, tl.n0 + c, row0, tl.g);
          } else {
            if (!GROUP_K && a.R != nullptr && row0 + lane < a.c_rows) {
              // residual row chunk (N % 32 == 0 is checked on the host), added in fp32
              const int4* rr = reinterpret_cast<const int4*>(static_cast<const __nv_bfloat16*>(a.R) +
                                                             static_cast<int64_t>(row0 + lane) * a.ldr + tl.n0 + c);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int4 q4 = rr[j];
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&q4);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const float2 f = __bfloat1622float2(h2[i]);
                  r[8 * j + 2 * i] = __float_as_uint(__uint_as_float(r[8 * j + 2 * i]) + f.x);
                  r[8 * j + 2 * i + 1] = __float_as_uint(__uint_as_float(r[8 * j + 2 * i + 1]) + f.y);
                }
              }
            }
            uint32_t v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = pack_bf16(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
            store_box(&tmC, [&](uint8_t* sl) { put_row_bf16(sl, lane, v); }, tl.n0 + c, row0, tl.g);
          }
        }
      }
      if (have) {
        tc_fence_before();
        mbar_arrive(&tempty[b]);
        ++acc;
      }
    }
    if (lane == 0) bulk_wait<0>();  // this warp's stores are complete before the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ----------------------------------------------------------------------------- host side
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    AT_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// 2-D bf16 row-major [rows, cols] (row stride ld elements), boxes of box_rows x 64, 128B swizzle.
CUtensorMap make_map(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(r));
  return m;
}

// 3-D bf16 [G, K, N] (N contiguous): boxes of 64 (N) x BK (K) x 1, 128B swizzle. K past the
// end of one group reads as zeros instead of the next group's first rows.
CUtensorMap make_map_kn(const void* base, int64_t G, int64_t K, int64_t N) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((N * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(G)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(N * 2), static_cast<cuuint64_t>(K * N * 2)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(BK), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3-D) failed: ", static_cast<int>(r));
  return m;
}

// Output map for the epilogue's 32 x 32 boxes. 2-D [rows, cols] (row stride ld) or, with
// groups > 0, 3-D [groups, rows, cols] (group stride rows * ld) so a partial box never
// writes into the next group. fp32 boxes have 128-byte rows (SWIZZLE_128B), bf16 boxes
// 64-byte rows (SWIZZLE_64B).
CUtensorMap make_out_map(void* base, bool f32, int64_t rows, int64_t cols, int64_t ld, int64_t groups) {
  const int64_t es = f32 ? 4 : 2;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "output base must be 16-byte aligned");
  TORCH_CHECK((ld * es) % 16 == 0, "output row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  const cuuint32_t rank = groups > 0 ? 3 : 2;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(groups > 0 ? groups : 1)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * es), static_cast<cuuint64_t>(rows * ld * es)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encoder()(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, base,
                         dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                         CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (output) failed: ", static_cast<int>(r));
  return m;
}

// 2-D one-byte [rows, cols] (row stride ld bytes), boxes of box_rows x 128 bytes, 128B swizzle.
CUtensorMap make_map_u8(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(ld % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK8), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (u8) failed: ", static_cast<int>(r));
  return m;
}

template <bool GROUP_K, int BN, int STAGES, int EPI, int LAYOUT, bool FP8 = false>
void launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mh,
            const Args& a, int grid, cudaStream_t stream) {
  constexpr size_t smem = 1024 + STAGES * Smem<BN>::kStageBytes + kEpiBytes +
                          (FP8 ? STAGES * sf_stage_bytes<BN>() : 0) + (2 * STAGES + 5) * 8 + 16;
  auto kfn = grouped_gemm_kernel<GROUP_K, BN, STAGES, EPI, LAYOUT, FP8>;
  static std::atomic<uint64_t> seen{0};
  AT_CUDA_CHECK(set_smem_limit_once(seen, kfn, static_cast<int>(smem)));
  kfn<<<grid, kThreads, smem, stream>>>(ma, mb, mc, mh, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gemm

// C[rows, N] = A[rows, K] @ B[g]^T per expert segment (offsets on rows, multiples of 128).
// epilogue: 0 = bf16 C, 1 = fp32 C, 2 = SwiGLU (H = silu(gate) * up, C = pre-activation or none)
// b_kn: B is [G, K, N] (N contiguous, e.g. the forward weight read as its transpose)
// instead of [G, N, K].
void grouped_gemm_m(const at::Tensor& A, const at::Tensor& B, const at::Tensor& offsets, const OptTensor& C,
                    const OptTensor& Hout, int64_t epilogue, at::Tensor error, int64_t num_sms, double timeout_s,
                    bool b_kn, const OptTensor& residual) {
  using namespace gemm;
  const c10::cuda::CUDAGuard guard(A.device());
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "A, B must be bf16");
  TORCH_CHECK(A.dim() == 2 && A.stride(1) == 1 && B.dim() == 3 && B.is_contiguous(),
              "A [rows, K], B [G, N, K] (or [G, K, N] with b_kn)");
  TORCH_CHECK(offsets.scalar_type() == at::kLong && offsets.numel() == B.size(0) + 1 && B.size(0) <= 1024,
              "offsets must be [G + 1] int64, G <= 1024");
  Args a{};
  a.G = static_cast<int>(B.size(0));
  a.N = static_cast<int>(b_kn ? B.size(2) : B.size(1));
  a.K = static_cast<int>(b_kn ? B.size(1) : B.size(2));
  a.M = static_cast<int>(A.size(0));
  TORCH_CHECK(A.size(1) == a.K && a.K % 8 == 0, "K mismatch / K % 8");
  TORCH_CHECK(!b_kn || a.N % 64 == 0, "an MN-major B needs N % 64 == 0");
  a.offsets = offsets.data_ptr<int64_t>();
  a.error = reinterpret_cast<uint32_t*>(error.data_ptr<int32_t>());
  a.timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  const CUtensorMap ma = make_map(A.data_ptr(), A.size(0), a.K, A.stride(0), BM);
  const CUtensorMap mb = b_kn ? make_map_kn(B.data_ptr(), a.G, a.K, a.N)
                              : make_map(B.data_ptr(), int64_t(a.G) * a.N, a.K, a.K, 256);
  a.c_rows = A.size(0);
  if (epilogue == kEpiSwiGLU) {
    TORCH_CHECK(a.N % 256 == 0 && Hout.has_value(), "SwiGLU needs N % 256 == 0 and an H output");
    a.H = Hout->data_ptr();
    a.ldh = Hout->stride(0);
    TORCH_CHECK(Hout->size(0) >= A.size(0), "H needs as many rows as A");
  }
  if (C.has_value()) {
    TORCH_CHECK(C->size(0) >= A.size(0) && C->stride(1) == 1, "C needs at least as many rows as A");
    TORCH_CHECK((epilogue == kEpiF32) == (C->scalar_type() == at::kFloat), "C dtype does not match the epilogue");
    a.C = C->data_ptr();
    a.ldc = C->stride(0);
  } else {
    TORCH_CHECK(epilogue == kEpiSwiGLU, "C is required");
  }
  if (residual.has_value()) {
    TORCH_CHECK(epilogue == kEpiBF16 && residual->scalar_type() == at::kBFloat16 && residual->stride(1) == 1 &&
                    residual->size(0) >= a.c_rows && residual->size(1) == a.N && a.N % 32 == 0 &&
                    (reinterpret_cast<uintptr_t>(residual->data_ptr()) & 15) == 0 && residual->stride(0) % 8 == 0,
                "residual: bf16 [rows, N] with N % 32 == 0, 16-byte aligned rows, bf16 epilogue");
    a.R = residual->data_ptr();
    a.ldr = residual->stride(0);
  }
  // output maps: rows past A's (the padding of the last segment) are clipped by the map
  const CUtensorMap mh = epilogue == kEpiSwiGLU ? make_out_map(a.H, false, a.c_rows, a.N / 2, a.ldh, 0)
                                                : CUtensorMap{};
  const CUtensorMap mc = a.C ? make_out_map(a.C, epilogue == kEpiF32, a.c_rows, a.N, a.ldc, 0) : mh;
  const int sms = num_sms > 0 ? static_cast<int>(num_sms) : at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (b_kn) {
    if (epilogue == kEpiBF16) launch<false, 256, 4, kEpiBF16, 2>(ma, mb, mc, mh, a, sms, stream);
    else if (epilogue == kEpiF32) launch<false, 256, 4, kEpiF32, 2>(ma, mb, mc, mh, a, sms, stream);
    else launch<false, 256, 4, kEpiSwiGLU, 2>(ma, mb, mc, mh, a, sms, stream);
  } else {
    if (epilogue == kEpiBF16) launch<false, 256, 4, kEpiBF16, 0>(ma, mb, mc, mh, a, sms, stream);
    else if (epilogue == kEpiF32) launch<false, 256, 4, kEpiF32, 0>(ma, mb, mc, mh, a, sms, stream);
    else launch<false, 256, 4, kEpiSwiGLU, 0>(ma, mb, mc, mh, a, sms, stream);
  }
}

// C[g] (M x N) = A[:, seg_g] @ B[:, seg_g]^T with A [M, tokens], B [N, tokens] (offsets on tokens),
// or, with tok_major, A [tokens, M] and B [tokens, N] (the activations as they are).
void grouped_gemm_k(const at::Tensor& A, const at::Tensor& B, const at::Tensor& offsets, at::Tensor C,
                    at::Tensor error, int64_t num_sms, double timeout_s, bool tok_major) {
  using namespace gemm;
  const c10::cuda::CUDAGuard guard(A.device());
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "A, B must be bf16");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1,
              "A [M, tokens], B [N, tokens] (or [tokens, M], [tokens, N] with tok_major)");
  TORCH_CHECK(C.dim() == 3 && C.is_contiguous(), "C must be [G, M, N]");
  Args a{};
  a.G = static_cast<int>(C.size(0));
  a.M = static_cast<int>(tok_major ? A.size(1) : A.size(0));
  a.N = static_cast<int>(tok_major ? B.size(1) : B.size(0));
  TORCH_CHECK(!tok_major || (a.M % 64 == 0 && a.N % 64 == 0 && A.size(0) == B.size(0)),
              "token-major operands need M, N multiples of 64 and the same token count");
  TORCH_CHECK(C.size(1) == a.M && C.size(2) == a.N && offsets.numel() == a.G + 1 && a.G <= 1024, "shape mismatch");
  a.offsets = offsets.data_ptr<int64_t>();
  a.C = C.data_ptr();
  a.ldc = a.N;
  a.c_group_stride = int64_t(a.M) * a.N;
  a.error = reinterpret_cast<uint32_t*>(error.data_ptr<int32_t>());
  a.timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  // token-major: boxes of 64 (M or N) x BK tokens, one per 64-wide MN atom
  const CUtensorMap ma = tok_major ? make_map(A.data_ptr(), A.size(0), a.M, A.stride(0), BK)
                                   : make_map(A.data_ptr(), a.M, A.size(1), A.stride(0), BM);
  const CUtensorMap mb = tok_major ? make_map(B.data_ptr(), B.size(0), a.N, B.stride(0), BK)
                                   : make_map(B.data_ptr(), a.N, B.size(1), B.stride(0), 256);
  TORCH_CHECK(C.scalar_type() == at::kFloat || C.scalar_type() == at::kBFloat16, "C must be fp32 or bf16");
  const bool f32 = C.scalar_type() == at::kFloat;
  const CUtensorMap mc = make_out_map(a.C, f32, a.M, a.N, a.N, a.G);
  const int sms = num_sms > 0 ? static_cast<int>(num_sms) : at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (tok_major) {
    if (f32) launch<true, 256, 4, kEpiF32, 3>(ma, mb, mc, mc, a, sms, stream);
    else launch<true, 256, 4, kEpiBF16, 3>(ma, mb, mc, mc, a, sms, stream);
  } else {
    if (f32) launch<true, 256, 4, kEpiF32, 0>(ma, mb, mc, mc, a, sms, stream);
    else launch<true, 256, 4, kEpiBF16, 0>(ma, mb, mc, mc, a, sms, stream);
  }
}

// Scale tiles for the fp8 GEMM: scales [groups * rows, KB] fp32 (powers of two) ->
// [groups, ceil(rows / 128), KB] tiles of 128 words; word (r % 32) * 4 + r / 32 holds row r's
// UE8M0 exponent in all four bytes (after a 32x128b copy: TMEM lane r % 32 of every
// subpartition, column r / 32). Rows past a group's `rows` read as scale 1.
__global__ void sf_tiles_kernel(const float* __restrict__ sc, int64_t ld, int64_t rows, int64_t tiles, int KB,
                                uint32_t* __restrict__ out, int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int w = static_cast<int>(i & 127);
    const int64_t tk = i >> 7;          // (group, row tile, kb)
    const int kb = static_cast<int>(tk % KB);
    const int64_t gt = tk / KB;
    const int64_t tile = gt % tiles, g = gt / tiles;
    const int64_t r = tile * 128 + (w >> 2) + 32 * (w & 3);
    const float v = r < rows ? sc[(g * rows + r) * ld + kb] : 1.f;
    out[i] = ((__float_as_uint(v) >> 23) & 0xFFu) * 0x01010101u;
  }
}

at::Tensor sf_tiles(const at::Tensor& sc, int64_t groups, int64_t rows_per_group) {
  // sc: [groups * rows_per_group, KB] fp32 -> uint8 [groups, ceil(rows_per_group / 128), KB, 512]
  TORCH_CHECK(sc.scalar_type() == at::kFloat && sc.dim() == 2 && unit_inner(sc) &&
                  sc.size(0) == groups * rows_per_group,
              "scales must be [groups * rows, KB] fp32");
  const int KB = static_cast<int>(sc.size(1));
  const int64_t tiles = (rows_per_group + 127) / 128;
  auto out = at::empty({groups, tiles, KB, 512}, sc.options().dtype(at::kByte));
  const int64_t total = groups * tiles * KB * 128;
  if (total == 0) return out;
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, 8192));
  sf_tiles_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      sc.data_ptr<float>(), sc.stride(0), rows_per_group, tiles, KB, reinterpret_cast<uint32_t*>(out.data_ptr<uint8_t>()),
      total);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// fp8 block-scaled grouped GEMM (forward shape): C[seg_g] = dequant(A)[seg_g] @ dequant(B[g])^T with
// A [rows, K] e4m3 and B [G, N, K] e4m3, each with one power-of-two fp32 scale per (row,
// 128-channel K block): sa [rows, K/128], sb [G, N, K/128]. Scales must be exact powers of two
// (the tensor cores take them as UE8M0 exponents). Epilogues as grouped_gemm_m; the SwiGLU
// epilogue expects 64-row gate / up blocks (N tiles of 128).
void grouped_gemm_fp8_m(const at::Tensor& A, const at::Tensor& sa, const at::Tensor& B, const at::Tensor& sb,
                        const at::Tensor& offsets, const OptTensor& C, const OptTensor& Hout, int64_t epilogue,
                        at::Tensor error, int64_t num_sms, double timeout_s) {
  using namespace gemm;
  const c10::cuda::CUDAGuard guard(A.device());
  TORCH_CHECK(A.element_size() == 1 && B.element_size() == 1, "A, B must be one-byte (e4m3) tensors");
  TORCH_CHECK(A.dim() == 2 && A.stride(1) == 1 && B.dim() == 3 && B.is_contiguous(), "A [rows, K], B [G, N, K]");
  TORCH_CHECK(offsets.scalar_type() == at::kLong && offsets.numel() == B.size(0) + 1 && B.size(0) <= 1024,
              "offsets must be [G + 1] int64, G <= 1024");
  Args a{};
  a.G = static_cast<int>(B.size(0));
  a.N = static_cast<int>(B.size(1));
  a.K = static_cast<int>(B.size(2));
  a.M = static_cast<int>(A.size(0));
  TORCH_CHECK(A.size(1) == a.K && a.K % 128 == 0, "K mismatch, or K not a multiple of 128");
  const int64_t KB = a.K / 128;
  TORCH_CHECK(sa.scalar_type() == at::kByte ||
                  (sa.scalar_type() == at::kFloat && sa.dim() == 2 && sa.size(0) == A.size(0) && sa.size(1) == KB &&
                   unit_inner(sa)),
              "sa must be [rows, K/128] fp32 (or its scale tiles)");
  TORCH_CHECK(sb.scalar_type() == at::kByte ||
                  (sb.scalar_type() == at::kFloat && sb.is_contiguous() && sb.numel() == int64_t(a.G) * a.N * KB),
              "sb must be [G, N, K/128] fp32 (or its scale tiles)");
  // scale tiles: given (uint8 [.., 512]) or built here from the fp32 scales
  at::Tensor ta = sa.scalar_type() == at::kByte ? sa : sf_tiles(sa, 1, A.size(0));
  at::Tensor tb = sb.scalar_type() == at::kByte ? sb : sf_tiles(sb.view({int64_t(a.G) * a.N, KB}), a.G, a.N);
  TORCH_CHECK(ta.numel() == (A.size(0) + 127) / 128 * KB * 512 && tb.numel() == int64_t(a.G) * ((a.N + 127) / 128) * KB * 512,
              "scale tiles have the wrong size");
  a.sfa_tiles = ta.data_ptr<uint8_t>();
  a.sfb_tiles = tb.data_ptr<uint8_t>();
  a.offsets = offsets.data_ptr<int64_t>();
  a.error = reinterpret_cast<uint32_t*>(error.data_ptr<int32_t>());
  a.timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  constexpr int BN8 = 128;
  const CUtensorMap ma = make_map_u8(A.data_ptr(), A.size(0), a.K, A.stride(0), BM);
  const CUtensorMap mb = make_map_u8(B.data_ptr(), int64_t(a.G) * a.N, a.K, a.K, BN8);
  a.c_rows = A.size(0);
  if (epilogue == kEpiSwiGLU) {
    TORCH_CHECK(a.N % BN8 == 0 && Hout.has_value(), "SwiGLU needs N % 128 == 0 and an H output");
    a.H = Hout->data_ptr();
    a.ldh = Hout->stride(0);
    TORCH_CHECK(Hout->size(0) >= A.size(0), "H needs as many rows as A");
  }
  if (C.has_value()) {
    TORCH_CHECK(C->size(0) >= A.size(0) && C->stride(1) == 1, "C needs at least as many rows as A");
    TORCH_CHECK((epilogue == kEpiF32) == (C->scalar_type() == at::kFloat), "C dtype does not match the epilogue");
    a.C = C->data_ptr();
    a.ldc = C->stride(0);
  } else {
    TORCH_CHECK(epilogue == kEpiSwiGLU, "C is required");
  }
  const CUtensorMap mh = epilogue == kEpiSwiGLU ? make_out_map(a.H, false, a.c_rows, a.N / 2, a.ldh, 0)
                                                : CUtensorMap{};
  const CUtensorMap mc = a.C ? make_out_map(a.C, epilogue == kEpiF32, a.c_rows, a.N, a.ldc, 0) : mh;
  const int sms = num_sms > 0 ? static_cast<int>(num_sms) : at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (epilogue == kEpiBF16) launch<false, BN8, 6, kEpiBF16, 0, true>(ma, mb, mc, mh, a, sms, stream);
  else if (epilogue == kEpiF32) launch<false, BN8, 6, kEpiF32, 0, true>(ma, mb, mc, mh, a, sms, stream);
  else launch<false, BN8, 6, kEpiSwiGLU, 0, true>(ma, mb, mc, mh, a, sms, stream);
}

}  // namespace b200ep
