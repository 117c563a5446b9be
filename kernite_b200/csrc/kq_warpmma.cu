// kq_warpmma.cu -- the Q4_K / Q6_K matvec for batch 1..8 with the multiply-adds on the tensor
// cores through warp-level MMA: at batch 1 (the default) integer MMAs (mma.sync m16n8k32, the
// raw quants as u8 A operands, x as three signed byte limbs, s32 accumulate), at batch 2..8 f16
// MMAs (m16n8k16, f16 operands from registers, f32 accumulate). The notes below describe the
// f16 variant; the integer variant's are at q6i8_half and q4i8_block.
//
// y[b, r] = sum_k W[r, k] * x[b, k], W in GGML k-quant blocks (144-byte Q4_K, 210-byte Q6_K).
//
// Why warp-level MMA for a matvec: the work is HBM-bound, and what limits a CUDA-core kernel is
// the instruction count per weight (every 4- or 6-bit quant has to become its own f32 before an
// FMA). Here a thread turns two quants into one f16x2 MMA operand register with one LOP3 (the
// 1024 + q magic) and one HFMA2 that applies the sub-block scale exactly, and the tensor core does
// the products. The A operand comes straight from registers, which tcgen05.mma cannot take (its A
// lives in shared or tensor memory, which would add a write and a read of 2 bytes per weight).
//
// Shape (one persistent CTA per SM, contiguous rows per CTA):
//  * A producer warp streams tiles of 16 rows x up to 16 super-blocks into a ring of shared
//    memory slots: one 1-D bulk copy for a tile of whole rows; for K-tiled rows one 3-D TMA copy
//    of a tensor map over W per band of 16 whole rows (the tensor-map tiles), else one bulk copy
//    per row segment. An mbarrier per slot counts the bytes in; Q6_K blocks at any even offset
//    need nothing special (readers use the byte offset from the aligned copy).
//  * A consumer warp takes one super-block of a tile: 16 MMAs (K = 16 each) over the tile's
//    16 rows (warp w takes block w, in a loop with the block's constants hoisted, when the tiles
//    are whole rows on 16-byte boundaries or tensor-map tiles; else 19 warps take turns over a
//    tile's blocks).
//    The 16 rows are the MMA's M, x (with the batch) is its N. Thread (g, c) of the
//    warp builds the A registers of rows g and g+8 from the bytes of its quarter of the block
//    (Q4_K: qs chunk c = sub-blocks 2c, 2c+1; Q6_K: sub-blocks c and c+4 of each half).
//  * The order of K inside an MMA is free as long as A and B agree, so each thread pairs the
//    nibbles its LOP3 masks give it, and x is laid out to match: at the start of the kernel every
//    CTA converts x into a table of MMA B fragments in shared memory.
//  * x goes in as an f16 pair hi + lo (hi = f16(x), lo = f16(x - hi)) in two B columns, so the
//    products carry ~22 bits of x: batch <= 4 fits one n8 MMA (column 2b + part), batch 5..8
//    takes two (hi, lo). x is first scaled by a power of two (per vector, undone at the end) when
//    its largest entry is at or above 2^10 (Q4_K) / 2^14 (Q6_K), or below 1, so that f16 never
//    overflows (Q4_K's sub-block sums of x included) and small vectors do not sink into f16
//    subnormals.
//  * Q4_K: A = q*sc exactly (integers <= 945), D = sum q*sc*x; the min term sum_j m_j X_j
//    (X_j = sum of x over sub-block j) is one more MMA per block with A = m_j; then
//    y += d*D - dmin*Dmin in f32.
//  * Q6_K (batch 1): A = q - 32 exactly; the 8 columns of the MMA separate the 8 sub-blocks of a
//    half block (B[k][n] = x_k if k lies in sub-block n, else 0), so D[row][n] = sum over
//    sub-block n of (q-32)*x and the int8 scales are applied in f32: y += d * sum_n sc_n D_n.
//    x enters as hi only here (no column is left for lo): relative error <= 2^-11 per product,
//    inside the 1e-3 * sum|w x| bound with room to spare, because Q6_K has no min term.
//  * Lanes' partial rows go to shared memory per band of 16 rows; every few bands the warps
//    meet at a barrier and sum them in a fixed order (deterministic), then write y.
//
// The GGML block layouts and the decode follow the public format (the CPU restatement in
// oracle/kq_oracle.c); the pattern "one output row per group of lanes, FMA chain over k" is the
// matvec of fxeqxmulfx/kernite's examples/microgpt/src/gpu.rs:100-131, re-shaped for HBM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>

#include <algorithm>
#include <string>
#include <type_traits>

#include "kq_device.cuh"
#include "kq_internal.h"

namespace kq {
// Device code and kernels in a named namespace: their mangled names are the same in this build
// and in the separately compiled module image (kq_module_image), where a caller looks them up.
namespace wm {

// Consumer warps: 19 + the producer = 5 warps per scheduler, which leaves 96 registers a thread
// (each scheduler's register file holds 16K: 5 x 32 x 96 <= 16384; 6 warps would leave 80).
constexpr uint32_t kMaxWarps = 19;
constexpr uint32_t kTileBlocks = 16;  // super-blocks of a K-tile, at most
constexpr uint32_t kTileRows = 16;    // rows of a tile = the MMA's M
constexpr uint32_t kRedBudget = 16384;  // bytes of shared memory for partial rows
// Q4_K table: bytes per (block, n-tile, column): 16 MMAs x 4 threads x 8 bytes, plus 32 bytes
// of padding so that the columns' rows start on different banks.
constexpr uint32_t kNStride = 16 * 32 + 32;
constexpr uint32_t kZeroBytes = 1024 + 64;
// The gap before rows 8..15 of a split tile: a Q4_K thread reads 16 bytes at 32-byte strides
// (16 + 32c), which fill half the banks; a row 16 bytes (mod 32) further fills the other half.
constexpr uint32_t kSplitGap = 16;  // covers every MMA offset of one block's fragments

// A descriptor flag bit outside the public KQ_FLAG_* set: batch 1 on the f16 warp-MMA variant
// instead of the integer one, so both stay reachable for tests and A/B timing. The integer
// variant is the default for both types (measured on B200: 10% faster for Q6_K, 1% for Q4_K,
// and its 24-bit fixed-point x is the more accurate).
constexpr uint32_t kFlagAltBatch1 = 1u << 30;
// Another such bit: the other choice of consumer warps (one per super-block of the widest K-tile,
// or kMaxWarps taking turns) for A/B timing.
constexpr uint32_t kFlagWarpPerBlock = 1u << 29;

// A chain launch: at most this many jobs (their parameters travel in the launch), and pushes to
// at most this many GPUs.
constexpr uint32_t kChainMaxJobs = 8;
constexpr uint32_t kChainMaxRanks = 8;

constexpr uint32_t kMagic = 0x64006400u;  // f16x2 (1024, 1024): OR a 10-bit field in = 1024 + v

struct WarpMmaArgs {
  const uint8_t* W;
  const float* x;
  float* y;
  unsigned* err;
  uint64_t ldx, ldy;
  uint64_t total_bytes, row_bytes;
  uint32_t rows, nb, batch;
  uint32_t nkt;          // K-tiles per band (super-blocks split as evenly as possible)
  uint32_t nw;           // consumer warps (at least the super-blocks of the widest K-tile)
  uint32_t ring, slot_bytes, seg_bytes;  // seg_bytes: shared-memory pitch of a tile's rows
  uint32_t table_off, mtable_off, ublk_off, zero_off, red_off, bars_off;  // shared-memory layout
  uint32_t zero;         // 0: multipliers built from it are opaque to the compiler
  uint32_t row_perm;     // 1: MMA row pairs are tile rows two apart (see pg)
  uint32_t split_tile;   // 1: whole-row tile in two copies, rows 8..15 kSplitGap bytes further
  uint32_t fixed_blocks; // 1: integer path with warp w fixed to block w (whole 16-byte rows)
  uint32_t ncol;         // B columns in use per n-tile
  uint32_t fb;           // bands of partial rows kept before a flush
  uint32_t ksplit;       // CTAs sharing each row range, each its 1/ksplit of the K-tiles (1: none)
  uint32_t row_unit, prologue, epilogue, flags;
  float eps, pair_scale;
  // 1: the tiles of whole bands come in by the tensor map (one 3-D TMA copy of 16 rows), rows
  // tile_pitch bytes apart; a CTA's last band of fewer than 16 rows still goes row by row, at the
  // same pitch
  uint32_t tmap_mode, tile_pitch;
  // 0, or the first K-tile of x's second part: the x table holds the K-tiles [0, xpart) first,
  // then [xpart, nkt), rebuilt in between by each warp for its own block (Q6_K tensor-map tiles
  // whose whole table would leave room for only two ring slots); every band's partial rows are
  // kept across the two parts
  uint32_t xpart;
  CUtensorMap tmap;  // W as [rows][super-blocks][block bytes] (Q6_K: [rows][8-block groups][1680 B])
};

// A matvec that is one job of a chain (one launch running several matvecs of one type and k in
// turn, each reading the previous one's output): the wait before its x is read, where its outputs
// go on the other GPUs of a row-sharded stack, and the counters that tell their readers the
// outputs are complete.
struct ChainSync {
  // null, or a counter on this GPU that must reach *epoch * wait_target before x is read
  const unsigned long long* wait_cnt;
  uint64_t wait_target;
  // outputs [0, push_rows) also go to push_y[p][o] for p < npush (0: they stay on this GPU)
  uint32_t npush, push_rows;
  float* push_y[kChainMaxRanks];
  // after its outputs are stored, each CTA adds its output count (pushed outputs when npush > 0)
  // to counter[p] for p < max(npush, 1); null counter[0]: no count
  unsigned long long* counter[kChainMaxRanks];
  // 1: push_y[p] are tagged vectors (8 bytes an element: the f32 value, then the tag of this
  // launch's outputs, WarpMmaShared::tag_out) and no counter is added to
  uint32_t tagged;
  uint32_t out_slot;  // tagged, split K: elements between the slots of the push_y vectors
};

// What one matvec has of its own when several share a launch's layout: its matrix, vectors and
// fused glue. (A lone launch takes these from its WarpMmaArgs.)
struct JobArgs {
  const uint8_t* W;
  const float* x;
  float* y;
  uint64_t total_bytes;
  uint32_t rows, row_unit, prologue, epilogue;
  float eps, pair_scale;
};

struct ChainParams {
  WarpMmaArgs lay;                  // the layout every job shares (its per-job fields unused)
  const unsigned long long* epoch;  // this GPU's token counter
  uint32_t njobs;
  JobArgs job[kChainMaxJobs];
  ChainSync sync[kChainMaxJobs];
};

// A lone matvec of a row-sharded stack (kq_matvec_push on the warp-MMA kernel): the push of its
// outputs to every rank and the counters, as a chain job has them, and its wait, whose target is
// (*epoch - 1) * wait_mul + wait_add.
struct PushArgs {
  ChainSync y;
  const unsigned long long* epoch;
  uint64_t wait_mul, wait_add;  // the counter's target, or with tagged x the tag x carries
  uint64_t push_mul, push_add;  // the tag of the outputs (tagged pushes)
  uint32_t x_slots;             // tagged x: its split-K slots (1: none)
  uint32_t reserved;
};

// The parts of shared memory that are not in the dynamic layout.
struct WarpMmaShared {
  int failed;
  double sq[kMaxWarps][8];  // [consumer warp][vector] sums of squares of x
  float ns[8];              // per vector: the RMS-norm factor (1 without norm)
  uint32_t tag_x, tag_out;  // tagged exchange: the tag x's elements must carry; the outputs' tag
  uint32_t x_slots;         // tagged x: the slots (split-K parts, K elements apart) summed per element
};

// Tiles the producer issues before it waits for the previous kernel to finish (when the consumers
// start loading x), in a CTA with at most kHoldMaxTiles tiles: the rest of the ring would queue
// ahead of those loads, and for a short matrix the x prologue is most of a launch's critical path.
// A long matrix keeps its whole head start.
constexpr uint32_t kHoldTiles = 2, kHoldMaxTiles = 16;

// The exponent e of a positive finite float v = f * 2^e, f in [0.5, 1) (frexpf's, for a normal v;
// for a subnormal v it gives -126, at or below which every caller clamps alike).
__device__ __forceinline__ int exponent_of(float v) {
  return static_cast<int>((__float_as_uint(v) >> 23) & 255u) - 126;
}

// 2^s as a float, s in [-126, 127].
__device__ __forceinline__ float pow2f(int s) { return __uint_as_float(static_cast<uint32_t>(s + 127) << 23); }

// 8 bytes of a tagged vector: the f32 value (low word) and its tag (high word), one aligned 8-byte
// load (so value and tag come from the same store), cached in L2 only: other GPUs' stores into
// this GPU's memory land in its L2, so a repeated load sees them, and the L1 (not coherent) is
// bypassed. (A system-scope load takes a slower path; the tag, not the load's scope, is what
// says the value is this step's.)
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}

// Two consecutive tagged elements (16-byte aligned) in one load; each 8-byte element is read whole.
__device__ __forceinline__ ulonglong2 ld_tagged2(const unsigned long long* p) {
  ulonglong2 v;
  asm volatile("ld.global.cg.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ void st_tagged(float* p, float v, uint32_t tag) {
  asm volatile("st.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag) : "memory");
}

// ---------------------------------------------------------------- register-level helpers

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;  // (a & b) | c
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// The low nibble of each byte from lo, the high nibble from hi (one LOP3).
__device__ __forceinline__ uint32_t nibble_select(uint32_t lo, uint32_t hi) {
  uint32_t d;  // (lo & 0x0F0F0F0F) | (hi & 0xF0F0F0F0)
  asm("lop3.b32 %0, %1, %2, %3, 0xB8;" : "=r"(d) : "r"(hi), "r"(0x0F0F0F0Fu), "r"(lo));
  return d;
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// x >> 8 and x >> (8 - s) as multiply-highs, x << s as a multiply: the same bits, computed on
// the FMA pipe, which the dequantisation leaves idle, instead of the ALU it saturates. The
// multipliers come in as values the compiler cannot see are powers of two.
__device__ __forceinline__ uint32_t mulhi(uint32_t x, uint32_t m) {
  uint32_t d;
  asm("mul.hi.u32 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(m));
  return d;
}
__device__ __forceinline__ uint32_t mullo(uint32_t x, uint32_t m) {
  uint32_t d;
  asm("mul.lo.u32 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(m));
  return d;
}

// 16 bytes at shared address `addr` as 4 words, for an address whose alignment class the whole
// warp shares: ALIGN 16, 8 or 4 loads directly; ALIGN 2 loads the 4-byte-aligned superset and
// funnel-shifts.
template <int ALIGN>
__device__ __forceinline__ void lds16(uint32_t addr, uint32_t (&w)[4]) {
  if constexpr (ALIGN == 16) {
    const uint4 v = lds_v4(addr);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (ALIGN == 8) {
    const uint2 v0 = lds_v2(addr), v1 = lds_v2(addr + 8);
    w[0] = v0.x; w[1] = v0.y; w[2] = v1.x; w[3] = v1.y;
  } else if constexpr (ALIGN == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = lds_u32(addr + 4 * i);
  } else {
    lds_words_unaligned<4>(addr, w);
  }
}

// D += A * B for one m16n8k16 tile (A row-major 16x16 f16, B column-major 16x8 f16, f32 D).
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The f16 part `hi` (p = 0) or `lo` (p = 1) of v: hi = f16(v), lo = f16(v - hi).
__device__ __forceinline__ __half part(float v, uint32_t p) {
  const __half h = __float2half_rn(v);
  if (p == 0) return h;
  return __float2half_rn(v - __half2float(h));
}

constexpr uint32_t f16x2_const(uint16_t lo, uint16_t hi) {
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// D += A * B for one m16n8k32 integer tile (A row-major 16x32 u8, B column-major 32x8 s8, s32 D).
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B + C for one m16n8k32 integer tile, C given apart from D (the first step of a sum).
__device__ __forceinline__ void imma16832_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, uint32_t b0, uint32_t b1, uint32_t c0,
                                            uint32_t c1, uint32_t c2, uint32_t c3) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%10, %11, %12, %13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}

// x as three signed byte limbs: v = L2 * 2^16 + L1 * 2^8 + L0 for an integer |v| <= 2^22.
__device__ __forceinline__ float limbs_to_f32(int l2, int l1, int l0) {
  return fmaf(static_cast<float>(l2), 65536.f, static_cast<float>(l1 * 256 + l0));
}

// A small unsigned integer (< 2^23) in byte 0..1 or 2..3 of w as an f32, without the XU pipe:
// the bytes go under the exponent of 2^23 and 2^23 comes off.
template <int HALF>
__device__ __forceinline__ float u16_to_f32(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, HALF ? 0x7432u : 0x7410u)) - 8388608.f;
}

// f16 bit patterns of the constants the decode uses
constexpr uint16_t kH1 = 0x3C00;        // 1.0
constexpr uint16_t kH16th = 0x2C00;     // 0.0625
constexpr uint16_t kHm64 = 0xD400;      // -64
constexpr uint16_t kHm96 = 0xD600;      // -96
constexpr uint16_t kHm1024 = 0xE400;    // -1024
constexpr uint16_t kHm1056 = 0xE420;    // -1056

// ---------------------------------------------------------------- Q6_K block

// 16 bytes at a 16-byte window offset, from the 32-byte aligned window [base, base + 32):
// words W..W+3 of it, funnel-shifted right by fs bits (0 or 16).
template <int W>
__device__ __forceinline__ void lds16_window(uint32_t base, uint32_t fs, uint32_t (&out)[4]) {
  const uint4 v0 = lds_v4(base), v1 = lds_v4(base + 16);
  const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) out[k] = __funnelshift_r(w[W + k], w[W + k + 1], fs);
}

// The quants of half hf of one Q6_K super-block for thread (g, c), rows g and g+8: L[row] = the
// 16 ql bytes at 64 hf + 16c, Q[row] = the 16 qh bytes at 128 + 32 hf + 16 (c & 1).
// MODE -1: every address 16-byte aligned; 4 or 8: aligned to that many bytes (direct loads);
// 0..3: all lanes share the offset 4 MODE + fs/8 within 16 bytes (two 16-byte loads and a funnel
// shift); -2: anything (4-byte loads and funnel shifts).
template <int MODE>
__device__ __forceinline__ void q6_load_half(uint32_t ag, uint32_t ah, uint32_t c, uint32_t hf,
                                             uint32_t fs, uint32_t (&L)[2][4], uint32_t (&Q)[2][4]) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint32_t base = r ? ah : ag;
    const uint32_t al = base + 64 * hf + 16 * c, aq = base + 128 + 32 * hf + 16 * (c & 1);
    if constexpr (MODE == -1) {
      lds16<16>(al, L[r]);
      lds16<16>(aq, Q[r]);
    } else if constexpr (MODE == 4 || MODE == 8) {
      lds16<MODE>(al, L[r]);
      lds16<MODE>(aq, Q[r]);
    } else if constexpr (MODE >= 0) {
      lds16_window<MODE>(al & ~15u, fs, L[r]);
      lds16_window<MODE>(aq & ~15u, fs, Q[r]);
    } else {
      lds16<2>(al, L[r]);
      lds16<2>(aq, Q[r]);
    }
  }
}

template <int MODE>
__device__ __forceinline__ void q6_load(uint32_t ag, uint32_t ah, uint32_t c, uint32_t fs,
                                        uint32_t (&L)[2][2][4], uint32_t (&Q)[2][2][4]) {
  q6_load_half<MODE>(ag, ah, c, 0, fs, L[0], Q[0]);
  q6_load_half<MODE>(ag, ah, c, 1, fs, L[1], Q[1]);
}

// 16 bytes at shared address `addr` whose residue mod 16 is known at compile time to be in
// the class F: 16 (0), 8 (8), 4 (4 or 12), 2 (2 or 10), 6 (6 or 14). Aligned classes load
// directly; for 2 and 6 the five 4-byte words from addr - 2 come in as 8- and 4-byte loads at
// their natural alignment and each output word is a 16-bit funnel shift of two of them.
template <int F>
__device__ __forceinline__ void lds16_class(uint32_t addr, uint32_t (&w)[4]) {
  if constexpr (F == 16 || F == 8 || F == 4) {
    lds16<F>(addr, w);
  } else {
    const uint32_t b = addr - 2;
    uint32_t v[5];
    if constexpr (F == 2) {  // b = 0 mod 8
      const uint2 p0 = lds_v2(b), p1 = lds_v2(b + 8);
      v[0] = p0.x; v[1] = p0.y; v[2] = p1.x; v[3] = p1.y; v[4] = lds_u32(b + 16);
    } else {                 // b = 4 mod 8
      const uint2 p1 = lds_v2(b + 4), p2 = lds_v2(b + 12);
      v[0] = lds_u32(b); v[1] = p1.x; v[2] = p1.y; v[3] = p2.x; v[4] = p2.y;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = __funnelshift_r(v[k], v[k + 1], 16);
  }
}

// The residue class (for lds16_class) of a 2-byte aligned offset o mod 16.
__host__ __device__ constexpr int residue_class(uint32_t o) {
  return (o & 15u) == 0 ? 16 : (o & 7u) == 0 ? 8 : (o & 3u) == 0 ? 4 : (o & 7u) == 2 ? 2 : 6;
}

// One half hf of a Q6_K super-block on the integer path, rows g and g+8 of thread (g, c):
// L[row] = the thread's 16 ql bytes, Q[row] = its 16 qh bytes. Per step, A = 4 + 4 6-bit quants
// of one sub-block (ql nibble | qh pair << 4, as bytes); B = the three byte limbs of the same
// elements of x (from the table, or zeros for lanes whose column is another sub-block); C of the
// first step = -32 * the limb sums of the thread's sub-blocks. Then y += d * sum_n sc_n D_n.
//  mkb: the accumulator start values of the block; bA, bB: this thread's B-fragment bases for
//  steps 0-1 and 2-3; sHi: the shift that brings the thread's qh pairs to bits 0-1 and 4-5;
//  k16, k28: 16 and 2^28 as values the compiler cannot see (x16 and >> 4 on the FMA pipe).
__device__ __forceinline__ void q6i8_half(uint32_t hf, const uint32_t (&L)[2][4],
                                          const uint32_t (&Q)[2][4], uint32_t ag, uint32_t ah,
                                          uint32_t c, uint32_t mkb, uint32_t bA, uint32_t bB,
                                          uint32_t k16, uint32_t k28, uint32_t sHi, float dg,
                                          float dh, float (&yacc)[2][2]) {
  int acc[3][4];
  uint2 ci[3];
#pragma unroll
  for (int l = 0; l < 3; ++l) ci[l] = lds_v2(mkb + hf * 96 + l * 32);
  const uint32_t bAh = bA + hf * 384, bBh = bB + hf * 384;
  // V: the thread's two qh pairs of each element slot at bits 0-1 (low group) and 4-5 (high
  // group) of each byte: qh bits 0-1 / 4-5 for c < 2, 2-3 / 6-7 for c >= 2 (sHi = 0 or 2)
  uint32_t V[2][4];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int i = 0; i < 4; ++i) V[r][i] = (Q[r][i] >> sHi) & 0x33333333u;
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    const int w0 = 2 * (st & 1), w1 = w0 + 1;
    uint32_t a0, a1, a2, a3;
    if (st < 2) {
      // low nibble | pair from bits 0-1 of V, moved to bits 4-5
      a0 = nibble_select(L[0][w0], mullo(V[0][w0], k16));
      a1 = nibble_select(L[1][w0], mullo(V[1][w0], k16));
      a2 = nibble_select(L[0][w1], mullo(V[0][w1], k16));
      a3 = nibble_select(L[1][w1], mullo(V[1][w1], k16));
    } else {
      // high nibble | pair from bits 4-5 of V, in place
      a0 = nibble_select(mulhi(L[0][w0], k28), V[0][w0]);
      a1 = nibble_select(mulhi(L[1][w0], k28), V[1][w0]);
      a2 = nibble_select(mulhi(L[0][w1], k28), V[0][w1]);
      a3 = nibble_select(mulhi(L[1][w1], k28), V[1][w1]);
    }
    const uint32_t bb = (st < 2 ? bAh : bBh) + 24 * (st & 1);
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      const uint2 bf = lds_v2(bb + 8 * l);
      if (st == 0)
        imma16832_c(acc[l], a0, a1, a2, a3, bf.x, bf.y, ci[l].x, ci[l].y, ci[l].x, ci[l].y);
      else
        imma16832(acc[l], a0, a1, a2, a3, bf.x, bf.y);
    }
  }
  // columns 2c, 2c+1 = sub-blocks 2c, 2c+1 of this half: scales 8 hf + 2c, +1
  const uint32_t sg = lds_u16(ag + 192 + 8 * hf + 2 * c);
  const uint32_t sh = lds_u16(ah + 192 + 8 * hf + 2 * c);
  const float v0 = limbs_to_f32(acc[2][0], acc[1][0], acc[0][0]);
  const float v1 = limbs_to_f32(acc[2][1], acc[1][1], acc[0][1]);
  const float v2 = limbs_to_f32(acc[2][2], acc[1][2], acc[0][2]);
  const float v3 = limbs_to_f32(acc[2][3], acc[1][3], acc[0][3]);
  yacc[0][0] += dg * fmaf(static_cast<float>(static_cast<int8_t>(sg & 0xffu)), v0,
                          static_cast<float>(static_cast<int8_t>(sg >> 8)) * v1);
  yacc[1][0] += dh * fmaf(static_cast<float>(static_cast<int8_t>(sh & 0xffu)), v2,
                          static_cast<float>(static_cast<int8_t>(sh >> 8)) * v3);
}

// One Q6_K super-block of rows g (at shared address ag) and g+8 (ah) for thread (g, c) of a warp,
// from its quants L, Q: 16 MMAs, A = q - 32 exactly (lo halves hold 1024 + q, hi halves
// 1024 + 16 q), the eight MMA columns being the eight 16-element sub-blocks of a half; then
// y += d * sum_n sc_n D_n.
__device__ __forceinline__ void q6_block(uint32_t ag, uint32_t ah, uint32_t c, uint32_t tab_kb,
                                         uint32_t k24, uint32_t kT, uint32_t kT13, float dg,
                                         float dh, const uint32_t (&L)[2][2][4],
                                         const uint32_t (&Q)[2][2][4], float (&yacc)[2][2]) {
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int o = 0; o < 2; ++o) {
        // byte pairs (0, 2) for o = 0, (1, 3) for o = 1
        const uint32_t Lg = o ? mulhi(L[hf][0][i], k24) : L[hf][0][i];
        const uint32_t Lh = o ? mulhi(L[hf][1][i], k24) : L[hf][1][i];
        const uint32_t Tg = o ? mulhi(Q[hf][0][i], kT13) : mullo(Q[hf][0][i], kT);
        const uint32_t Th = o ? mulhi(Q[hf][1][i], kT13) : mullo(Q[hf][1][i], kT);
        const uint32_t lo_g = lop_and_or(Lg, 0x000F000Fu, lop_and_or(Tg, 0x00300030u, kMagic));
        const uint32_t lo_h = lop_and_or(Lh, 0x000F000Fu, lop_and_or(Th, 0x00300030u, kMagic));
        const uint32_t hi_g = lop_and_or(Lg, 0x00F000F0u, lop_and_or(Tg, 0x03000300u, kMagic));
        const uint32_t hi_h = lop_and_or(Lh, 0x00F000F0u, lop_and_or(Th, 0x03000300u, kMagic));
        const uint32_t a0 = hadd2(lo_g, f16x2_const(kHm1056, kHm1056));
        const uint32_t a1 = hadd2(lo_h, f16x2_const(kHm1056, kHm1056));
        const uint32_t a2 = hfma2(hi_g, f16x2_const(kH16th, kH16th), f16x2_const(kHm96, kHm96));
        const uint32_t a3 = hfma2(hi_h, f16x2_const(kH16th, kH16th), f16x2_const(kHm96, kHm96));
        const uint2 bf = lds_v2(tab_kb + (hf * 8 + 2 * i + o) * 64);
        if (o == 0)
          mma16816(acc0, a0, a1, a2, a3, bf.x, bf.y);
        else
          mma16816(acc1, a0, a1, a2, a3, bf.x, bf.y);
      }
    }
    // columns 2c, 2c+1 = sub-blocks 2c, 2c+1 of this half: scales 8 hf + 2c, +1
    const uint32_t sg = lds_u16(ag + 192 + 8 * hf + 2 * c);
    const uint32_t sh = lds_u16(ah + 192 + 8 * hf + 2 * c);
    const float sg0 = static_cast<float>(static_cast<int8_t>(sg & 0xffu));
    const float sg1 = static_cast<float>(static_cast<int8_t>(sg >> 8));
    const float sh0 = static_cast<float>(static_cast<int8_t>(sh & 0xffu));
    const float sh1 = static_cast<float>(static_cast<int8_t>(sh >> 8));
    yacc[0][0] += dg * fmaf(sg0, acc0[0] + acc1[0], sg1 * (acc0[1] + acc1[1]));
    yacc[1][0] += dh * fmaf(sh0, acc0[2] + acc1[2], sh1 * (acc0[3] + acc1[3]));
  }
}

// One Q4_K super-block on the integer path, rows g and g+8 of thread (g, c). Thread c owns qs
// chunk c (sub-blocks 2c: low nibbles, 2c+1: high). 8 steps (o, i): nibble o of bytes 8i..8i+7
// of the chunk, i.e. elements 64c + 32o + 8i .. +7, whose x limbs are table chunk 8c + 4o + i;
// the lanes of MMA column n = 2c + o read them (b0, b1: this thread's bases for o = 0, 1, or
// the zero region), so column n sums sub-block n. Then y += d sum sc_n D_n - dmin sum m_n X_n.
//  sel_sc, m_lo, m_hi, sh_m: the thread's 6-bit scale/min unpack; X: the sums of x (limb units)
//  over sub-blocks 2c, 2c+1; u0: the block's 2^-shift of x.
// Q5K: the Q5_K block (176 bytes: qh[32] at 16, qs at 48), whose fifth bit of element 32g + l is
// bit g of qh[l]: the thread's elements 64c + 32o + b take bit 2c + o of qh[b], and qh word j
// holds the same byte positions b as qs word j of the chunk.
template <bool Q5K = false>
__device__ __forceinline__ void q4i8_block(uint32_t ag, uint32_t ah, uint32_t c, uint32_t b0,
                                           uint32_t b1, uint32_t k28, uint32_t sel_sc,
                                           uint32_t m_lo, uint32_t m_hi, uint32_t sh_m, float2 X,
                                           float u0, float (&yacc)[2][2]) {
  constexpr uint32_t kQs = Q5K ? 48 : 16;
  // one accumulator set per nibble (o): two independent chains of four MMAs per limb
  int acc[2][3][4];
  const uint4 hg = lds_v4(ag), hh = lds_v4(ah);
  uint32_t Wg[8], Wh[8];
  {
    const uint4 g0 = lds_v4(ag + kQs + 32 * c), g1 = lds_v4(ag + kQs + 16 + 32 * c);
    const uint4 h0 = lds_v4(ah + kQs + 32 * c), h1 = lds_v4(ah + kQs + 16 + 32 * c);
    Wg[0] = g0.x; Wg[1] = g0.y; Wg[2] = g0.z; Wg[3] = g0.w;
    Wg[4] = g1.x; Wg[5] = g1.y; Wg[6] = g1.z; Wg[7] = g1.w;
    Wh[0] = h0.x; Wh[1] = h0.y; Wh[2] = h0.z; Wh[3] = h0.w;
    Wh[4] = h1.x; Wh[5] = h1.y; Wh[6] = h1.z; Wh[7] = h1.w;
  }
  // Q5_K: the thread's two fifth bits of each byte position at bits 0 (o = 0) and 1 (o = 1)
  uint32_t Vg[8], Vh[8];
  if constexpr (Q5K) {
    const uint4 p0 = lds_v4(ag + 16), p1 = lds_v4(ag + 32);
    const uint4 q0 = lds_v4(ah + 16), q1 = lds_v4(ah + 32);
    const uint32_t pg[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    const uint32_t ph[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      Vg[j] = (pg[j] >> (2 * c)) & 0x03030303u;
      Vh[j] = (ph[j] >> (2 * c)) & 0x03030303u;
    }
  }
  // nibble o of word w, with (Q5_K) the fifth bit from v moved to bit 4 of each byte
  auto quant = [&](uint32_t w, uint32_t v, int o) {
    const uint32_t nib = (o ? mulhi(w, k28) : w) & 0x0F0F0F0Fu;
    if constexpr (Q5K) return lop_and_or(o ? (v << 3) : (v << 4), 0x10101010u, nib);
    return nib;
  };
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int o = 0; o < 2; ++o) {
      const uint32_t a0 = quant(Wg[2 * i], Q5K ? Vg[2 * i] : 0u, o);
      const uint32_t a1 = quant(Wh[2 * i], Q5K ? Vh[2 * i] : 0u, o);
      const uint32_t a2 = quant(Wg[2 * i + 1], Q5K ? Vg[2 * i + 1] : 0u, o);
      const uint32_t a3 = quant(Wh[2 * i + 1], Q5K ? Vh[2 * i + 1] : 0u, o);
      const uint32_t bb = (o ? b1 : b0) + 24 * i;
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        const uint2 bf = lds_v2(bb + 8 * l);
        if (i == 0)
          imma16832_c(acc[o][l], a0, a1, a2, a3, bf.x, bf.y, 0u, 0u, 0u, 0u);
        else
          imma16832(acc[o][l], a0, a1, a2, a3, bf.x, bf.y);
      }
    }
  // scales and mins of sub-blocks 2c, 2c+1 (the thread's columns) as floats
  auto scm = [&](const uint4& hd, float& s0, float& s1, float& m0, float& m1) {
    const uint32_t ts = __byte_perm(hd.w, hd.y, sel_sc);
    const uint32_t sc16 = (ts & m_lo) | ((ts >> 10) & m_hi);
    const uint32_t tm = __byte_perm(hd.w, hd.z, sel_sc);
    const uint32_t m16 = ((tm >> sh_m) & m_lo) | ((tm >> 10) & m_hi);
    s0 = u16_to_f32<0>(sc16);
    s1 = u16_to_f32<1>(sc16);
    m0 = u16_to_f32<0>(m16);
    m1 = u16_to_f32<1>(m16);
  };
  float sg0, sg1, mg0, mg1, sh0, sh1, mh0, mh1;
  scm(hg, sg0, sg1, mg0, mg1);
  scm(hh, sh0, sh1, mh0, mh1);
  const float dg = u0 * h2f(hg.x & 0xffffu), dmg = u0 * h2f(hg.x >> 16);
  const float dh = u0 * h2f(hh.x & 0xffffu), dmh = u0 * h2f(hh.x >> 16);
  // column 2c (sub-block 2c) is summed by the o = 0 MMAs alone, column 2c + 1 by the o = 1 ones
  const float v0 = limbs_to_f32(acc[0][2][0], acc[0][1][0], acc[0][0][0]);
  const float v1 = limbs_to_f32(acc[1][2][1], acc[1][1][1], acc[1][0][1]);
  const float v2 = limbs_to_f32(acc[0][2][2], acc[0][1][2], acc[0][0][2]);
  const float v3 = limbs_to_f32(acc[1][2][3], acc[1][1][3], acc[1][0][3]);
  yacc[0][0] += dg * fmaf(sg0, v0, sg1 * v1) - dmg * fmaf(mg0, X.x, mg1 * X.y);
  yacc[1][0] += dh * fmaf(sh0, v2, sh1 * v3) - dmh * fmaf(mh0, X.x, mh1 * X.y);
}

// ---------------------------------------------------------------- the kernels' parts

// The rows [r_begin, r_end) of a matvec that this CTA streams and multiplies: a contiguous share
// of whole output units (pairs of rows for the product epilogues).
// With split K (ksplit > 1), CTAs ksplit * g .. ksplit * g + ksplit - 1 share row range g.
__device__ __forceinline__ void cta_rows(const JobArgs& v, uint32_t ksplit, uint32_t& r_begin,
                                         uint32_t& r_end) {
  const uint64_t units = v.rows / v.row_unit;
  const uint32_t groups = gridDim.x / ksplit, g = blockIdx.x / ksplit;
  r_begin = static_cast<uint32_t>(units * g / groups) * v.row_unit;
  r_end = static_cast<uint32_t>(units * (g + 1) / groups) * v.row_unit;
}

// The K-tiles [kt_lo, kt_hi) of each band that this CTA takes: all, or with split K its share.
__device__ __forceinline__ void cta_ktiles(uint32_t nkt, uint32_t ksplit, uint32_t& kt_lo,
                                           uint32_t& kt_hi) {
  const uint32_t part = blockIdx.x % ksplit;
  kt_lo = part * nkt / ksplit;
  kt_hi = (part + 1) * nkt / ksplit;
}

// A lone launch's per-matvec fields.
__device__ __forceinline__ JobArgs job_of(const WarpMmaArgs& a) {
  return JobArgs{a.W, a.x, a.y, a.total_bytes, a.rows, a.row_unit, a.prologue, a.epilogue, a.eps,
                 a.pair_scale};
}

// The 128-byte aligned start of the dynamic shared memory.
__device__ __forceinline__ uint8_t* smem_base(uint8_t* smem) {
  return smem + ((128u - (smem_u32(smem) & 127u)) & 127u);
}

// Thread 0 sets up the ring's mbarriers (a full and an empty one per slot); the CTA then meets.
__device__ __forceinline__ void init_ring(const WarpMmaArgs& a, uint8_t* base, WarpMmaShared& sh) {
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + a.bars_off);
  if (threadIdx.x == 0) {
    sh.failed = 0;
    for (uint32_t s = 0; s < a.ring; ++s) {
      mbar_init(smem_u32(&bars[s]), 1);
      mbar_init(smem_u32(&bars[a.ring + s]), a.nw);
    }
    fence_mbar_init();
  }
  __syncthreads();
}

// A 3-D tiled TMA copy of box (x, y, z) of `tmap` (a kernel parameter) into shared `dst`,
// completing on `bar`; no multicast.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tmap, uint32_t x, uint32_t y,
                                            uint32_t z, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}

// The producer warp's part of one matvec: the tiles of this CTA's rows, each into the next ring
// slot once the consumers have freed it. Lane r of the warp copies row r of a tile (16 rows, one
// bulk copy each, at the padded pitch), or lane 0 the tile's rows in one copy; lane 0 posts the
// tile's byte count on its slot's mbarrier. s, phase: the ring position, carried from one matvec
// of a launch to the next; issued: the tiles this warp issued before in the launch (the first
// `ring` of them need no free slot). Returns false once a wait gave up.
template <int QT, bool XP = false>
__device__ __forceinline__ bool produce_job(const WarpMmaArgs& a, const JobArgs& v, uint8_t* base,
                                            WarpMmaShared& sh, uint32_t& s, uint32_t& phase,
                                            uint32_t& issued) {
  constexpr uint32_t kBlk = QT == 4 ? kQ4KBytes : QT == 5 ? kQ5KBytes : kQ6KBytes;
  int& s_failed = sh.failed;
  const uint32_t ring_s = smem_u32(base);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + a.bars_off);
  auto full_bar = [&](uint32_t s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](uint32_t s) { return smem_u32(&bars[a.ring + s]); };
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t RB = a.row_bytes;
  uint32_t r_begin, r_end;
  cta_rows(v, a.ksplit, r_begin, r_end);
  const uint32_t nbands = (r_end - r_begin + kTileRows - 1) / kTileRows;
  uint32_t kt_lo, kt_hi;
  cta_ktiles(a.nkt, a.ksplit, kt_lo, kt_hi);
  const uint32_t nktc = kt_hi - kt_lo;
  const uint32_t ntiles = nbands * nktc;
  const uint64_t pol = policy_evict_first();
  const uint64_t end_floor = v.total_bytes & ~uint64_t(15);
  for (uint32_t t = 0; t < ntiles; ++t) {
    // hold until the previous kernel is done, when the consumers load x (a no-op when the
    // weights are not static: the producer has waited for it already)
    if (issued == kHoldTiles && issued < a.ring && ntiles <= kHoldMaxTiles) pdl_wait();
    if (issued >= a.ring) {
      int ok = 1;
      if (lane == 0) {
        if (*reinterpret_cast<volatile int*>(&s_failed)) {
          ok = 0;
        } else if (!mbar_wait_sleep(empty_bar(s), phase ^ 1)) {
          s_failed = 1;
          report_error(a.err, kErrWaitEmpty);
          ok = 0;
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
    }
    // band by band, K-tile by K-tile; with x in two parts, every band's K-tiles of the first
    // part, then every band's of the second (the consumers' order)
    uint32_t band, kt;
    if constexpr (!XP) {
      band = t / nktc, kt = kt_lo + t % nktc;
    } else if (t < nbands * a.xpart) {
      band = t / a.xpart, kt = t % a.xpart;
    } else {
      const uint32_t u = t - nbands * a.xpart, w = a.nkt - a.xpart;
      band = u / w, kt = a.xpart + u % w;
    }
    const uint32_t r0 = r_begin + band * kTileRows;
    const uint32_t r1 = min(r0 + kTileRows, r_end);
    const uint32_t slot = ring_s + s * a.slot_bytes;
    // K-tile kt: super-blocks [kc0, kc1), kq + (kt < kr) of them (the consumers' split)
    const uint32_t kq = a.nb / a.nkt, kr = a.nb % a.nkt;
    const uint32_t kc0 = kt * kq + min(kt, kr), kc1 = kc0 + kq + (kt < kr ? 1u : 0u);
    if (a.tmap_mode && r1 - r0 == kTileRows) {
      // a whole band by the tensor map, one copy
      if (lane == 0) {
        mbar_arrive_expect_tx(full_bar(s), kTileRows * a.tile_pitch);
        tma_load_3d(slot, &a.tmap, 0, QT == 6 ? kc0 / 8 : kc0, r0, full_bar(s), pol);  // Q6_K: groups
      }
      __syncwarp();
      ++issued;
      if (++s == a.ring) {
        s = 0;
        phase ^= 1;
      }
      continue;
    }
    const uint32_t r = r0 + lane;
    uint64_t a0 = 0, a1 = 0;
    if (a.seg_bytes == 0) {
      // whole rows: one copy of the tile's 16-byte-aligned superset, by lane 0
      if (lane == 0) {
        a0 = (uint64_t(r0) * RB) & ~uint64_t(15);
        a1 = (uint64_t(r1) * RB + 15) & ~uint64_t(15);
        if (a1 > end_floor) {
          for (uint64_t i = end_floor; i < v.total_bytes; i += 2)
            sts_u16(slot + static_cast<uint32_t>(i - a0),
                    __ldg(reinterpret_cast<const unsigned short*>(v.W + i)));
          a1 = end_floor;
        }
        if (a1 < a0) a1 = a0;
      }
    } else if (lane < kTileRows && r < r1) {
      const uint64_t b0 = uint64_t(r) * RB + uint64_t(kc0) * kBlk;
      const uint64_t b1 = uint64_t(r) * RB + uint64_t(kc1) * kBlk;
      a0 = b0 & ~uint64_t(15);
      a1 = (b1 + 15) & ~uint64_t(15);
      if (a1 > end_floor) {
        // the end of W is off a 16-byte boundary: its last bytes (an even count, < 16) are
        // read with plain loads
        const uint32_t dst = slot + lane * a.seg_bytes;
        for (uint64_t i = end_floor; i < v.total_bytes; i += 2)
          sts_u16(dst + static_cast<uint32_t>(i - a0),
                  __ldg(reinterpret_cast<const unsigned short*>(v.W + i)));
        a1 = end_floor;
      }
      if (a1 < a0) a1 = a0;
    }
    uint32_t bytes = static_cast<uint32_t>(a1 - a0), total = bytes;
#pragma unroll
    for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    __syncwarp();
    if (lane == 0) mbar_arrive_expect_tx(full_bar(s), total);
    __syncwarp();
    if (a.tmap_mode) {
      // a band of fewer than 16 rows: row by row at the tensor-map layout's pitch (the rows start
      // on 16-byte boundaries, so each copy is exactly the row's K-tile)
      if (bytes) bulk_g2s(slot + lane * a.tile_pitch, v.W + a0, bytes, full_bar(s), pol);
    } else if (a.split_tile) {
      // rows r0..r0+7 at the slot, rows r0+8.. kSplitGap bytes past where they would follow
      // (rows are whole and start on 16-byte boundaries here, so a1 - a0 = (r1 - r0) * RB)
      if (lane == 0 && bytes) {
        const uint32_t first = static_cast<uint32_t>(std::min<uint64_t>(bytes, 8 * RB));
        bulk_g2s(slot, v.W + a0, first, full_bar(s), pol);
        if (bytes > first)
          bulk_g2s(slot + first + kSplitGap, v.W + a0 + first, bytes - first, full_bar(s), pol);
      }
    } else if (bytes) {
      bulk_g2s(slot + lane * a.seg_bytes, v.W + a0, bytes, full_bar(s), pol);
    }
    // (whole-row tiles: only lane 0 has bytes, and its destination is the slot itself)
    ++issued;
    if (++s == a.ring) {
      s = 0;
      phase ^= 1;
    }
  }
  return true;
}

// The consumer warps' part of one matvec: x into the B-fragment table (with the RMS-norm sums),
// then every tile of this CTA's rows from the ring, MMAs, and the outputs. s, phase: the ring
// position, carried from one matvec of a launch to the next. sync: null for a lone matvec; for a
// job of a chain, where its outputs are also pushed.
template <int QT, int NT, bool HILO, bool I8, int TXS = 0, int PART = 0>
__device__ __forceinline__ void consume_job(const WarpMmaArgs& a, const JobArgs& mj,
                                            const ChainSync* sync, uint8_t* base,
                                            WarpMmaShared& sh, uint32_t& s, uint32_t& phase,
                                            uint32_t opq = 0) {
  constexpr uint32_t kBlk = QT == 4 ? kQ4KBytes : QT == 5 ? kQ5KBytes : kQ6KBytes;
  constexpr int kTarget = QT == 4 ? 10 : 14;  // x is scaled so that max |x| < 2^kTarget
  // x: plain f32 (TXS 0), a tagged vector (1), or a tagged vector of several split-K slots (2)
  constexpr bool TX = TXS > 0;
  int& s_failed = sh.failed;
  double (&s_sq)[kMaxWarps][8] = sh.sq;
  float (&s_ns)[8] = sh.ns;

  const uint32_t ring_s = smem_u32(base);
  const uint32_t table_s = ring_s + a.table_off;
  const uint32_t mtable_s = ring_s + a.mtable_off;
  float* ublk = reinterpret_cast<float*>(base + a.ublk_off);  // [vector][block]: 2^-shift of x
  const uint32_t ublk_s = ring_s + a.ublk_off;
  // (the tile loops read it, and the sums of x, with explicit shared-memory loads)
  auto ublk_at = [&](uint32_t i) { return __uint_as_float(lds_u32(ublk_s + 4 * i)); };
  float* red = reinterpret_cast<float*>(base + a.red_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + a.bars_off);
  auto full_bar = [&](uint32_t s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](uint32_t s) { return smem_u32(&bars[a.ring + s]); };

  const uint32_t nw = a.nw;
  const uint32_t nthr = nw * 32;
  // opq: 0, read anew for each job of a chain, so that nothing derived from the thread index is
  // hoisted out of the chain's job loop (held in registers through the x prologue)
  const uint32_t tx = threadIdx.x + opq;
  const uint32_t warp = tx >> 5, lane = tx & 31;
  const uint64_t RB = a.row_bytes;
  uint32_t r_begin, r_end;
  cta_rows(mj, a.ksplit, r_begin, r_end);
  const uint32_t nbands = (r_end - r_begin + kTileRows - 1) / kTileRows;

  const uint32_t tid = tx;  // 0 .. nthr-1
  const uint32_t g = lane >> 2, c = lane & 3;
  const uint32_t B = a.batch;

  // ---- x prologue, one pass. Each warp takes 256-element blocks of x (one super-block of one
  // vector: an "x-block"), four at a time with all 32 loads of a lane in flight. Per x-block:
  //  * the sum of squares (f64, for the RMS norm, which is a scalar and is applied to y at the
  //    end) and max |x|;
  //  * a power of two s for the block: 1 when max |x| is in [1, 2^kTarget), else the one that
  //    brings it just under 2^kTarget (f16 never overflows, Q4_K's sub-block sums of x included;
  //    tiny blocks do not sink into f16 subnormals; small-integer inputs stay exact); 1/s is
  //    kept for the fix-up;
  //  * the scaled values, split into f16 parts, go to their places in the B-fragment table;
  //  * Q4_K: the sums of its eight 32-element sub-blocks (a reduce-scatter by shuffles).
  {
    if constexpr (PART == 2) __syncwarp();  // (this warp's reads of its first-part entries first)
    if (lane == 0)
      for (int b = 0; b < 8; ++b) s_sq[warp][b] = 0.0;
    if constexpr (I8) {
      // Batch 1, integer table, of the x-blocks [kb_lo, kb_hi) at entries kb - kb_lo (the scales
      // of x, ublk, at kb). Lane l owns the 8 consecutive elements 8l .. 8l+7 of an x-block,
      // which are chunk l of the block's table entry (the 8 bytes of each limb), so its loads
      // are two 16-byte ones (four for a tagged x), its table writes three 8-byte ones, and the
      // per-sub-block sums need two shuffles. kXG x-blocks per round, all loads in flight.
      // PART 0: all of x; 1, 2: the first or second part (warp w builds x-blocks w, w + nw, ...,
      // with nw the K-tile's blocks: the ones it reads in the fixed-block loop)
      const uint32_t kb_lo = PART == 2 ? a.xpart * (a.nb / a.nkt) : 0u;
      const uint32_t kb_hi = PART == 1 ? a.xpart * (a.nb / a.nkt) : a.nb;
      constexpr int kXG = TX ? 4 : 6;  // (more would spill: a tagged x doubles the live loads)
      const uint32_t want_tag = TX ? sh.tag_x : 0u;
      const uint32_t x_slots = TXS == 2 ? sh.x_slots : 1u;
      const uint64_t kx = uint64_t(a.nb) * kQK;  // elements between x's slots
      for (uint32_t xb0 = kb_lo + warp; xb0 < kb_hi; xb0 += kXG * nw) {
        float v[kXG][8];
        bool tags_ok = true;
#pragma unroll
        for (int j = 0; j < kXG; ++j) {
          const uint32_t kb = xb0 + j * nw;
          if (kb < kb_hi) {
            if constexpr (TX) {
              const unsigned long long* src =
                  reinterpret_cast<const unsigned long long*>(mj.x) + kb * kQK + 8 * lane;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const ulonglong2 w = ld_tagged2(src + 2 * q);
                v[j][2 * q] = __uint_as_float(static_cast<uint32_t>(w.x));
                v[j][2 * q + 1] = __uint_as_float(static_cast<uint32_t>(w.y));
                tags_ok &= static_cast<uint32_t>(w.x >> 32) == want_tag &&
                           static_cast<uint32_t>(w.y >> 32) == want_tag;
              }
              // split-K slots 1.. of the writer: added in slot order (the same sum on every rank)
              if constexpr (TXS == 2)
              for (uint32_t sl = 1; sl < x_slots; ++sl) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const ulonglong2 w = ld_tagged2(src + uint64_t(sl) * kx + 2 * q);
                  v[j][2 * q] += __uint_as_float(static_cast<uint32_t>(w.x));
                  v[j][2 * q + 1] += __uint_as_float(static_cast<uint32_t>(w.y));
                  tags_ok &= static_cast<uint32_t>(w.x >> 32) == want_tag &&
                             static_cast<uint32_t>(w.y >> 32) == want_tag;
                }
              }
            } else {
              const float4* src = reinterpret_cast<const float4*>(mj.x + kb * kQK + 8 * lane);
              const float4 p0 = __ldcg(src), p1 = __ldcg(src + 1);
              v[j][0] = p0.x, v[j][1] = p0.y, v[j][2] = p0.z, v[j][3] = p0.w;
              v[j][4] = p1.x, v[j][5] = p1.y, v[j][6] = p1.z, v[j][7] = p1.w;
            }
          }
        }
        if constexpr (TX) {
          if (!tags_ok) {
            // some element is not this step's yet: wait for each, bounded (at once when this CTA
            // or an earlier launch already gave up); unrolled, so that v stays in registers
            uint64_t t0 = 0;
#pragma unroll
            for (int j = 0; j < kXG; ++j) {
              const uint32_t kb = xb0 + j * nw;
              if (kb >= kb_hi) break;
              const unsigned long long* src =
                  reinterpret_cast<const unsigned long long*>(mj.x) + kb * kQK + 8 * lane;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                float sum = 0.f;
                for (uint32_t sl = 0; sl < x_slots; ++sl) {
                  const unsigned long long* at = src + uint64_t(sl) * kx + i;
                  unsigned long long w = ld_tagged(at);
                  while (static_cast<uint32_t>(w >> 32) != want_tag) {
                    if (*reinterpret_cast<volatile int*>(&s_failed) ||
                        (a.err && *reinterpret_cast<volatile unsigned*>(a.err)))
                      break;
                    if (t0 == 0) t0 = globaltimer();
                    if (globaltimer() - t0 > kWaitBudgetNs) {
                      report_error(a.err, kErrWaitPeer);
                      s_failed = 1;
                      break;
                    }
                    w = ld_tagged(at);
                  }
                  sum = sl ? sum + __uint_as_float(static_cast<uint32_t>(w))
                           : __uint_as_float(static_cast<uint32_t>(w));
                }
                v[j][i] = sum;
              }
            }
          }
        }
#pragma unroll
        for (int j = 0; j < kXG; ++j) {
          const uint32_t kb = xb0 + j * nw;
          if (kb >= kb_hi) break;
          float mx = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[j][i]));
#pragma unroll
          for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          double sq = 0.0;  // only the RMS norm needs it
          if (mj.prologue == KQ_PROLOGUE_RMSNORM) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              sq = fma(static_cast<double>(v[j][i]), static_cast<double>(v[j][i]), sq);
#pragma unroll
            for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
          }
          // 24-bit fixed point for the block: the power of two that brings max |x| into
          // [2^21, 2^22), so that x = (L2 2^16 + L1 2^8 + L0) 2^-sh with signed byte limbs
          // |L2| <= 64, |L1|, |L0| <= 128 (an integer-valued x stays exact).
          int e = 1;
          if (mx > 0.f && isfinite(mx)) e = exponent_of(mx);  // mx = f * 2^e, f in [0.5, 1)
          const int shv = mx > 0.f ? max(-126, min(126, 22 - e)) : 0;
          const float sc = pow2f(shv);
          if (lane == 0) {
            s_sq[warp][0] += sq;
            ublk[kb] = pow2f(-shv);
          }
          uint32_t pk[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};  // limb bytes, 4 to a word
          int tl[3] = {0, 0, 0};                              // per-limb sums (Q6_K)
          int tx = 0;                                         // sum of X (Q4_K, Q5_K)
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int X = __float2int_rn(v[j][i] * sc);
            const int l0 = ((X + 128) & 255) - 128;
            const int x1 = (X - l0) >> 8;
            const int l1 = ((x1 + 128) & 255) - 128;
            const int l2 = (x1 - l1) >> 8;
            const uint32_t sft = 8 * (i & 3);
            pk[0][i >> 2] |= (static_cast<uint32_t>(l0) & 0xffu) << sft;
            pk[1][i >> 2] |= (static_cast<uint32_t>(l1) & 0xffu) << sft;
            pk[2][i >> 2] |= (static_cast<uint32_t>(l2) & 0xffu) << sft;
            tl[0] += l0, tl[1] += l1, tl[2] += l2;
            tx += X;
          }
          // chunk `lane` of the block: 24 bytes, 8 of each limb
          const uint32_t at = table_s + ((kb - kb_lo) * 32 + lane) * 24;
#pragma unroll
          for (int l = 0; l < 3; ++l)
            asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(at + 8 * l), "r"(pk[l][0]), "r"(pk[l][1])
                         : "memory");
          if constexpr (QT == 6) {
            // C init of the MMAs: -32 * (sum of each limb over each 16-element sub-block), so that
            // A = q (unsigned) gives sum (q - 32) x exactly; sub-block sb is lanes 2 sb, 2 sb + 1.
            // Entry ((kb' * 2 + half) * 3 + l) * 8 + (sub-block within the half), kb' = kb - kb_lo.
            const uint32_t sb = lane >> 1;
#pragma unroll
            for (int l = 0; l < 3; ++l) {
              const int t = tl[l] + __shfl_xor_sync(0xffffffffu, tl[l], 1);
              if ((lane & 1) == 0)
                asm volatile("st.shared.s32 [%0], %1;" ::"r"(
                                 mtable_s + (((kb - kb_lo) * 2 + (sb >> 3)) * 24 + l * 8 + (sb & 7)) * 4),
                             "r"(-32 * t)
                             : "memory");
            }
          } else {
            // the sum of x (in limb units) over each 32-element sub-block, lanes 4 r .. 4 r + 3,
            // for the min term
            int t = tx + __shfl_xor_sync(0xffffffffu, tx, 1);
            t += __shfl_xor_sync(0xffffffffu, t, 2);
            if ((lane & 3) == 0)
              asm volatile("st.shared.f32 [%0], %1;" ::"r"(mtable_s + ((kb - kb_lo) * 8 + (lane >> 2)) * 4),
                           "f"(static_cast<float>(t))
                           : "memory");
          }
        }
      }
    } else {
    const uint32_t nxb = a.nb * B;
    for (uint32_t xb0 = warp; xb0 < nxb; xb0 += 4 * nw) {
      float v[4][8];
      bool tags_ok = true;
      const uint32_t want_tag = TX ? sh.tag_x : 0u;
      const uint32_t x_slots = TXS == 2 ? sh.x_slots : 1u;
      const uint64_t kx = uint64_t(a.nb) * kQK;  // elements between x's slots
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t xb = xb0 + j * nw;
        if (xb < nxb) {
          const uint32_t b = xb / a.nb, kb = xb - b * a.nb;
          if constexpr (TX) {
            // a tagged vector (batch 1): the values, and whether every tag is this step's; the
            // loads of all four x-blocks are in flight together, the stale ones reloaded after
            const unsigned long long* src =
                reinterpret_cast<const unsigned long long*>(mj.x) + kb * kQK + lane;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              const unsigned long long w = ld_tagged(src + 32 * r);
              v[j][r] = __uint_as_float(static_cast<uint32_t>(w));
              tags_ok &= static_cast<uint32_t>(w >> 32) == want_tag;
            }
            // split-K slots 1.. of the writer: added in slot order (the same sum on every rank)
            if constexpr (TXS == 2)
            for (uint32_t sl = 1; sl < x_slots; ++sl) {
#pragma unroll
              for (int r = 0; r < 8; ++r) {
                const unsigned long long w = ld_tagged(src + uint64_t(sl) * kx + 32 * r);
                v[j][r] += __uint_as_float(static_cast<uint32_t>(w));
                tags_ok &= static_cast<uint32_t>(w >> 32) == want_tag;
              }
            }
          } else {
            const float* src = mj.x + b * a.ldx + kb * kQK + lane;
#pragma unroll
            for (int r = 0; r < 8; ++r) v[j][r] = __ldcg(src + 32 * r);
          }
        }
      }
      if constexpr (TX) {
        if (!tags_ok) {
          // some element is not this step's yet: wait for each, bounded (at once when this CTA
          // or an earlier launch already gave up)
          // (unrolled, so that v stays in registers; the code is cold)
          uint64_t t0 = 0;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t xb = xb0 + j * nw;
            if (xb >= nxb) break;
            const unsigned long long* src =
                reinterpret_cast<const unsigned long long*>(mj.x) + (xb % a.nb) * kQK + lane;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              float sum = 0.f;
              for (uint32_t sl = 0; sl < x_slots; ++sl) {
                const unsigned long long* at = src + uint64_t(sl) * kx + 32 * r;
                unsigned long long w = ld_tagged(at);
                while (static_cast<uint32_t>(w >> 32) != want_tag) {
                  if (*reinterpret_cast<volatile int*>(&s_failed) ||
                      (a.err && *reinterpret_cast<volatile unsigned*>(a.err)))
                    break;
                  if (t0 == 0) t0 = globaltimer();
                  if (globaltimer() - t0 > kWaitBudgetNs) {
                    report_error(a.err, kErrWaitPeer);
                    s_failed = 1;
                    break;
                  }
                  w = ld_tagged(at);
                }
                sum = sl ? sum + __uint_as_float(static_cast<uint32_t>(w)) : __uint_as_float(static_cast<uint32_t>(w));
              }
              v[j][r] = sum;
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t xb = xb0 + j * nw;
        if (xb >= nxb) break;
        const uint32_t b = xb / a.nb, kb = xb - b * a.nb;
        double sq = 0.0;  // only the RMS norm needs it
        float mx = 0.f;
#pragma unroll
        for (int r = 0; r < 8; ++r) mx = fmaxf(mx, fabsf(v[j][r]));
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (mj.prologue == KQ_PROLOGUE_RMSNORM) {
#pragma unroll
          for (int r = 0; r < 8; ++r)
            sq = fma(static_cast<double>(v[j][r]), static_cast<double>(v[j][r]), sq);
#pragma unroll
          for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        }
        {
          int e = 1;
          if (mx > 0.f && isfinite(mx)) e = exponent_of(mx);  // mx = f * 2^e, f in [0.5, 1)
          const int sh = (e > kTarget || e <= 0) ? max(-126, min(126, kTarget - e)) : 0;
          const float sc = pow2f(sh);
          if (lane == 0) {
            s_sq[warp][b] += sq;
            ublk[b * a.nb + kb] = pow2f(-sh);
          }
  #pragma unroll
          for (int r = 0; r < 8; ++r) v[j][r] *= sc;
          if constexpr (QT == 4) {
            // entry (kb, t, n, m, c), 8 bytes at ((kb NT + t) ncol + n) kNStride + 32 m + 8 c:
            // regs (b0b1, b2b3) of thread (g = n, c) in MMA m of block kb, n-tile t. For
            // MMA m = 2i + o, thread c holds b0b1 = x[64c + 4i + o], x[64c + 32 + 4i + o + 2] and
            // b2b3 = x[64c + 32 + 4i + o], x[64c + 4i + o + 2]: element 64c + 32 hb + 4i + w
            // (w = o + 2 s2) sits in reg hb ^ s2, half s2. Here element = 32 r + lane.
            const uint32_t i = (lane >> 2) & 7, w = lane & 3;
            const uint32_t o = w & 1, s2 = w >> 1;
            const uint32_t m = 2 * i + o;
  #pragma unroll
            for (int r = 0; r < 8; ++r) {
              const uint32_t c_r = r >> 1, hb = r & 1;
              const uint32_t within = 32 * m + 8 * c_r + (((hb ^ s2) << 2) | (s2 << 1));
  #pragma unroll
              for (uint32_t pp = 0; pp < (HILO ? 2u : 1u); ++pp) {
                const uint32_t t = (HILO && NT == 2) ? pp : 0u;
                const uint32_t n = HILO ? (NT == 1 ? 2 * b + pp : b) : b;
                sts_u16(table_s + ((kb * NT + t) * a.ncol + n) * kNStride + within,
                        __half_as_ushort(part(v[j][r], pp)));
              }
            }
            // sub-block sums X_r = sum over lanes of v[r]: reduce-scatter by lane bits 4, 3, 2,
            // then a butterfly over bits 1, 0; lane l ends with X_((l >> 2) & 7).
            float w4[4], w2[2];
            const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
  #pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float keep = b4 ? v[j][q + 4] : v[j][q], give = b4 ? v[j][q] : v[j][q + 4];
              w4[q] = keep + __shfl_xor_sync(0xffffffffu, give, 16);
            }
  #pragma unroll
            for (int q = 0; q < 2; ++q) {
              const float keep = b3 ? w4[q + 2] : w4[q], give = b3 ? w4[q] : w4[q + 2];
              w2[q] = keep + __shfl_xor_sync(0xffffffffu, give, 8);
            }
            float X = (b2 ? w2[1] : w2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? w2[0] : w2[1], 4);
            X += __shfl_xor_sync(0xffffffffu, X, 2);
            X += __shfl_xor_sync(0xffffffffu, X, 1);
            if ((lane & 3) == 0) {
              // min entry (kb, t, n, c), 4 bytes at ((kb NT + t) ncol + n) 16 + 4c: b0b1 of the min
              // MMA = (X_2c, X_2c+1) of vector b
              const uint32_t jj = (lane >> 2) & 7;
  #pragma unroll
              for (uint32_t pp = 0; pp < (HILO ? 2u : 1u); ++pp) {
                const uint32_t t = (HILO && NT == 2) ? pp : 0u;
                const uint32_t n = HILO ? (NT == 1 ? 2 * b + pp : b) : b;
                sts_u16(mtable_s + ((kb * NT + t) * a.ncol + n) * 16 + 4 * (jj >> 1) + 2 * (jj & 1),
                        __half_as_ushort(part(X, pp)));
              }
            }
          } else {
            // entry (kb, h, m, c, u) = 8 bytes, read by thread (g, c) with g & 3 == c and u = g >> 2:
            // u = 0: (pair of sub-block c, 0); u = 1: (0, pair of sub-block c + 4). Element
            // 128h + 64u + 16c + 4i + w (w = o + 2 s2, m = 2i + o) sits in reg u, half s2, and
            // the same half of the other reg is zero. Here element = 32 r + lane.
            const uint32_t i = (lane >> 2) & 3, w = lane & 3, o = w & 1, s2 = w >> 1;
  #pragma unroll
            for (int r = 0; r < 8; ++r) {
              const uint32_t h = r >> 2, u = (r >> 1) & 1, cc = ((r & 1) << 1) | (lane >> 4);
              const uint32_t ent = (((kb * 2 + h) * 8 + 2 * i + o) * 4 + cc) * 2 + u;
              sts_u16(table_s + ent * 8 + u * 4 + s2 * 2, __half_as_ushort(__float2half_rn(v[j][r])));
              sts_u16(table_s + ent * 8 + (u ^ 1) * 4 + s2 * 2, 0);
            }
          }

        }
      }
    }
    }
    // a zeroed region that lanes without a B column read their fragments from (the second part
    // of x has it already; its warps go on alone: each reads only the entries it built)
    if constexpr (PART != 2) {
      for (uint32_t i = tid; i < kZeroBytes / 4; i += nthr)
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(ring_s + a.zero_off + 4 * i), "r"(0u) : "memory");
      named_barrier(1, nthr);
    }
    if (PART != 2 && tid < B) {
      float ns = 1.f;
      if (mj.prologue == KQ_PROLOGUE_RMSNORM) {
        double t = 0.0;
        for (uint32_t w = 0; w < nw; ++w) t += s_sq[w][tid];
        ns = static_cast<float>(
            1.0 / sqrt(t / (static_cast<double>(a.nb) * kQK) + static_cast<double>(mj.eps)));
      }
      s_ns[tid] = ns;  // read at the flushes, which start with a barrier
    }
  }

  // ---- per-thread constants
  // Q4_K scale/min unpack (sub-blocks j = 2c, 2c+1; bytes p, p+1 of the header words)
  const uint32_t p = 2 * (c & 1);
  const bool upper = c >= 2;
  const uint32_t sel_sc = upper ? (p | ((4 + p) << 4) | ((p + 1) << 8) | ((5 + p) << 12))
                                : ((4 + p) | ((4 + p) << 4) | ((5 + p) << 8) | ((5 + p) << 12));
  const uint32_t m_lo = upper ? 0x000F000Fu : 0x003F003Fu;
  const uint32_t m_hi = upper ? 0x00300030u : 0u;
  const uint32_t sh_m = upper ? 4u : 0u;
  // Q6_K: the qh bit pairs of this thread's groups go to bits 4-5 / 8-9 of each byte pair, by a
  // shift of sT = 4 (c < 2) or 2 (c >= 2) for bytes 0, 2 and of 8 - sT right for bytes 1, 3
  // B-fragment table offsets of this thread; lanes without a column read the zero region
  const bool tab_on = QT == 4 ? (g < a.ncol) : ((g & 3) == c);
  const uint32_t tab_lane = QT == 4 ? g * kNStride + c * 8 : (c * 2 + (g >> 2)) * 8;
  const uint32_t zero_s = ring_s + a.zero_off + (QT != 6 ? c * 8 : 0);
  const uint32_t k24 = (1u << 24) << a.zero;              // >> 8
  const uint32_t k28 = (1u << 28) << a.zero;              // >> 4
  // I8 Q6_K: the shift of the thread's qh pairs (see q6i8_half), and 16 kept opaque
  const uint32_t k16 = 16u << a.zero;
  const uint32_t sHi = c >= 2 ? 2u : 0u;
  const uint32_t kT = (1u << (QT == 6 ? (c >= 2 ? 2 : 4) : 0)) << a.zero;    // << sT
  const uint32_t kT13 = (1u << (QT == 6 ? (c >= 2 ? 26 : 28) : 0)) << a.zero;  // >> (8 - sT)
  // MMA rows g and g+8 of this thread are tile rows pg and ph (= pg + 8, or pg + 4 in a split
  // tile). With whole-row tiles whose row pitch is 32 or 96 mod 128 bytes, MMA rows (0,1), (2,3),
  // ... are tile rows (0,2), (1,3), ..., 64 bytes apart mod 128, so the two rows of a
  // quarter-warp's 16-byte loads take disjoint banks. With a pitch of 0 mod 128 the tile is split
  // (rows 8..15 stored kSplitGap bytes further) and MMA rows (0,1), (2,3), ... are tile rows
  // (0,8), (1,9), ... for g < 8 and (4,12), (5,13), ... for g + 8.
  const uint32_t pg = a.split_tile ? ((g & 1) * 8 + (g >> 1))
                                   : a.row_perm ? ((g & 4) | ((g & 1) << 1) | ((g >> 1) & 1)) : g;
  const uint32_t ph = a.split_tile ? pg + 4 : pg + 8;
  // the vectors whose outputs this thread accumulates (Q4_K: c, or 2c and 2c+1; Q6_K: 0)
  const uint32_t vb0 = QT == 6 ? 0u : ((HILO && NT == 1) ? c : 2 * c);
  const uint32_t vb1 = min(vb0 + 1, B - 1);
  const uint32_t vb0c = min(vb0, B - 1);

  float yacc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // rows g, g+8 x this thread's vectors
  // Tiles are walked band by band, K-tile by K-tile, with no divisions: K-tile kt has
  // kq + (kt < kr) super-blocks (the producer splits the same way).
  const uint32_t nkt = a.nkt, kq = a.nb / nkt, kr = a.nb % nkt;
  const uint32_t rb32 = static_cast<uint32_t>(RB);
  // byte offsets of tile rows pg and ph in a whole-row slot (or a tensor-map slot, whose rows are
  // tile_pitch bytes apart)
  const uint32_t pitch = a.tmap_mode ? a.tile_pitch : rb32;
  const uint32_t pg_rb = pg * pitch + (a.split_tile && pg >= 8 ? kSplitGap : 0u);
  const uint32_t ph_rb = ph * pitch + (a.split_tile && ph >= 8 ? kSplitGap : 0u);
  // When every row starts on a 16-byte boundary, a block's offset within 16 bytes is the same
  // for all rows of a warp: (kb * block bytes) mod 16.
  const bool rows16 = (rb32 & 15u) == 0;
  // One Q4_K super-block on the f16 path (rows g and g+8 of the tile at ag, ah): tab_t, bm_at:
  // this thread's B-fragment and min-term addresses of the block (or the zero region); u0, u1:
  // the block's 2^-shift of x for the thread's vectors.
  auto q4f16_block = [&](uint32_t ag, uint32_t ah, const uint32_t (&tab_t)[NT],
                         const uint32_t (&bm_at)[NT], float u0, float u1) {
    const uint4 hg = lds_v4(ag), hh = lds_v4(ah);
    const uint4 qg0 = lds_v4(ag + 16 + 32 * c), qg1 = lds_v4(ag + 32 + 32 * c);
    const uint4 qh0 = lds_v4(ah + 16 + 32 * c), qh1 = lds_v4(ah + 32 + 32 * c);
    // scales -> S = (sc_lo, sc_hi/16), Z = (-1024 sc_lo, -64 sc_hi), their swaps, mins
    uint32_t Sg, Zg, S2g, Z2g, Amg, Sh, Zh, S2h, Z2h, Amh;
    auto prep = [&](const uint4& hd, uint32_t& S, uint32_t& Z, uint32_t& S2, uint32_t& Z2,
                    uint32_t& Am) {
      const uint32_t ts = __byte_perm(hd.w, hd.y, sel_sc);
      const uint32_t M = lop_and_or(ts, m_lo, lop_and_or(ts >> 10, m_hi, kMagic));
      S = hfma2(M, f16x2_const(kH1, kH16th), f16x2_const(kHm1024, kHm64));
      Z = hmul2(S, f16x2_const(kHm1024, kHm1024));
      S2 = __byte_perm(S, 0, 0x1032);
      Z2 = __byte_perm(Z, 0, 0x1032);
      const uint32_t tm = __byte_perm(hd.w, hd.z, sel_sc);
      const uint32_t Mm = lop_and_or(tm >> sh_m, m_lo, lop_and_or(tm >> 10, m_hi, kMagic));
      Am = hadd2(Mm, f16x2_const(kHm1024, kHm1024));
    };
    prep(hg, Sg, Zg, S2g, Z2g, Amg);
    prep(hh, Sh, Zh, S2h, Z2h, Amh);
    const uint32_t qg[8] = {qg0.x, qg0.y, qg0.z, qg0.w, qg1.x, qg1.y, qg1.z, qg1.w};
    const uint32_t qh[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
    float acc0[NT][4], acc1[NT][4], accm[NT][4];
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc0[tt][j] = acc1[tt][j] = accm[tt][j] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int o = 0; o < 2; ++o) {
        const uint32_t wg = o ? mulhi(qg[i], k24) : qg[i];
        const uint32_t wh = o ? mulhi(qh[i], k24) : qh[i];
        const uint32_t a0 = hfma2(lop_and_or(wg, 0x00F0000Fu, kMagic), Sg, Zg);
        const uint32_t a1 = hfma2(lop_and_or(wh, 0x00F0000Fu, kMagic), Sh, Zh);
        const uint32_t a2 = hfma2(lop_and_or(wg, 0x000F00F0u, kMagic), S2g, Z2g);
        const uint32_t a3 = hfma2(lop_and_or(wh, 0x000F00F0u, kMagic), S2h, Z2h);
        const uint32_t m = 2 * i + o;
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
          const uint2 bf = lds_v2(tab_t[tt] + 32 * m);
          if (o == 0)
            mma16816(acc0[tt], a0, a1, a2, a3, bf.x, bf.y);
          else
            mma16816(acc1[tt], a0, a1, a2, a3, bf.x, bf.y);
        }
      }
    }
    // the min term: A = (m_2c, m_2c+1) in slots 2c, 2c+1 of rows g, g+8
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) {
      const uint32_t bm = lds_u32(bm_at[tt]);
      mma16816(accm[tt], Amg, Amh, 0u, 0u, bm, 0u);
    }
    const float dg = h2f(hg.x & 0xffffu), dmg = h2f(hg.x >> 16);
    const float dh = h2f(hh.x & 0xffffu), dmh = h2f(hh.x >> 16);
    if constexpr (HILO && NT == 1) {
      // columns 2c (hi) and 2c+1 (lo) are vector c
      const float Dg = (acc0[0][0] + acc1[0][0]) + (acc0[0][1] + acc1[0][1]);
      const float Dh = (acc0[0][2] + acc1[0][2]) + (acc0[0][3] + acc1[0][3]);
      yacc[0][0] += u0 * (dg * Dg - dmg * (accm[0][0] + accm[0][1]));
      yacc[1][0] += u0 * (dh * Dh - dmh * (accm[0][2] + accm[0][3]));
    } else if constexpr (HILO) {
      // tile 0 hi, tile 1 lo; columns 2c, 2c+1 are vectors 2c, 2c+1
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float uj = j ? u1 : u0;
        const float Dg = (acc0[0][j] + acc1[0][j]) + (acc0[1][j] + acc1[1][j]);
        const float Dh = (acc0[0][2 + j] + acc1[0][2 + j]) + (acc0[1][2 + j] + acc1[1][2 + j]);
        yacc[0][j] += uj * (dg * Dg - dmg * (accm[0][j] + accm[1][j]));
        yacc[1][j] += uj * (dh * Dh - dmh * (accm[0][2 + j] + accm[1][2 + j]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float uj = j ? u1 : u0;
        yacc[0][j] += uj * (dg * (acc0[0][j] + acc1[0][j]) - dmg * accm[0][j]);
        yacc[1][j] += uj * (dh * (acc0[0][2 + j] + acc1[0][2 + j]) - dmh * accm[0][2 + j]);
      }
    }
  };
  // per-block constants of the f16 path
  auto q4f16_consts = [&](uint32_t kb, uint32_t (&tab_t)[NT], uint32_t (&bm_at)[NT], float& u0,
                          float& u1) {
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) {
      tab_t[tt] = tab_on ? table_s + (kb * NT + tt) * a.ncol * kNStride + tab_lane : zero_s;
      bm_at[tt] = tab_on ? mtable_s + ((kb * NT + tt) * a.ncol + g) * 16 + 4 * c : zero_s;
    }
    u0 = ublk_at(vb0c * a.nb + kb);
    u1 = ublk_at(vb1 * a.nb + kb);
  };

  // The band is done: this warp's partial rows go to the reduction buffer; every fb bands (and
  // after the last) the warps meet and sum them in a fixed order into y. With x in two parts
  // (PART 1, 2): the first stores the partial rows (no flush: fb covers every band), the second
  // adds to them.
  auto band_end = [&](uint32_t band, uint32_t& bi) {
    if constexpr (QT == 6 || I8) {
      // the four threads of a row hold different sub-blocks of vector 0
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        yacc[r][0] += __shfl_xor_sync(0xffffffffu, yacc[r][0], 1);
        yacc[r][0] += __shfl_xor_sync(0xffffffffu, yacc[r][0], 2);
      }
      if (c == 0) {
        float* rg = &red[((bi * nw + warp) * kTileRows + pg) * B];
        float* rh = &red[((bi * nw + warp) * kTileRows + ph) * B];
        if (PART == 2) {
          // (the first part's partial of the same row, written by this thread)
          *rg += yacc[0][0];
          *rh += yacc[1][0];
        } else {
          *rg = yacc[0][0];
          *rh = yacc[1][0];
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t b = (HILO && NT == 1) ? (j == 0 ? c : 8u) : 2 * c + j;
        if (b < B) {
          red[((bi * nw + warp) * kTileRows + pg) * B + b] = yacc[0][j];
          red[((bi * nw + warp) * kTileRows + ph) * B + b] = yacc[1][j];
        }
      }
    }
    yacc[0][0] = yacc[0][1] = yacc[1][0] = yacc[1][1] = 0.f;

    if (PART != 1 && (bi + 1 == a.fb || band + 1 == nbands)) {
      // Flush: sum every warp's partial of each row in a fixed order and write y.
      named_barrier(1, nthr);
      const uint32_t band0 = band - bi;
      const uint32_t R = mj.row_unit;
      const uint32_t nout = (bi + 1) * (kTileRows / R) * B;
      for (uint32_t o = tid; o < nout; o += nthr) {
        const uint32_t b = o % B;
        const uint32_t q = o / B;  // output index within the flushed bands
        const uint32_t row16 = (q % (kTileRows / R)) * R;
        const uint32_t bj = q / (kTileRows / R);
        const uint32_t row = r_begin + (band0 + bj) * kTileRows + row16;
        if (row >= r_end) continue;
        float v0 = 0.f;
        // (band-major, then warp, then row: the threads of a warp read consecutive rows)
        const float* rp = red + (bj * nw * kTileRows + row16) * B + b;
        for (uint32_t w = 0; w < nw; ++w) v0 += rp[w * kTileRows * B];
        v0 *= s_ns[b];
        uint32_t out = row;
        if (R != 1) {
          float v1 = 0.f;
          const float* rq = rp + B;
          for (uint32_t w = 0; w < nw; ++w) v1 += rq[w * kTileRows * B];
          v1 *= s_ns[b];
          v0 = pair_value(v0, v1, mj.epilogue, mj.pair_scale);
          out = row / 2;
        }
        // (with split K, v0 is this CTA's part of the sum over K: it goes to its own slot of
        // every rank's tagged vector only, where the reader adds the slots up)
        if (a.ksplit == 1) mj.y[b * a.ldy + out] = v0;
        // a chain job's pushed outputs also go to every rank's full vector (batch 1)
        if (sync && out < sync->push_rows) {
          if (sync->tagged) {
            const uint32_t tag = sh.tag_out;
            const uint32_t at = (blockIdx.x % a.ksplit) * sync->out_slot + out;
            for (uint32_t rk = 0; rk < sync->npush; ++rk) st_tagged(sync->push_y[rk] + 2 * at, v0, tag);
          } else {
            for (uint32_t rk = 0; rk < sync->npush; ++rk) sync->push_y[rk][out] = v0;
          }
        }
      }
      named_barrier(1, nthr);
      bi = 0;
    } else {
      ++bi;
    }
  };

  // Q6_K integer path, tiles of whole rows on 16-byte boundaries, one warp per block: warp w
  // takes block w of every tile, so its block's offset within 16 bytes (2w mod 16) is fixed, and
  // the loop is compiled once per residue class, with every address but the slot's hoisted.
  if constexpr (QT == 6 && I8 && TXS <= 1) {
    if (a.fixed_blocks && a.tmap_mode) {
      // Tensor-map tiles of K-tiled rows: warp w takes block w of every K-tile (whose 16-byte
      // residue, 2w mod 16, is the same in every tile); the x constants change with the K-tile.
      // (Compiled for lone launches and for push kernels whose tagged x has one slot.)
      const uint32_t fkb = warp;
      const uint32_t off_g = pg_rb + fkb * kBlk, off_h = ph_rb + fkb * kBlk;
      uint32_t kt_lo, kt_hi;
      cta_ktiles(nkt, a.ksplit, kt_lo, kt_hi);
      // the K-tiles [kt_a, kt_z) of every band (all, or with x in two parts those of the part),
      // whose x-blocks are the table's from kb_base on
      auto tmap_loop = [&](auto cls, uint32_t kt_a, uint32_t kt_z, uint32_t kb_base) {
        constexpr int F = decltype(cls)::value;
        uint32_t bi = 0;
        for (uint32_t band = 0; band < nbands; ++band) {
          for (uint32_t kt = kt_a; kt < kt_z; ++kt) {
            const uint32_t kb = kt * kq + fkb;
            const float u0 = ublk_at(kb);
            const uint32_t tkb = table_s + ((kb - kb_base) * 32 + 2 * c) * 24;
            const uint32_t bA = g == c ? tkb : zero_s;
            const uint32_t bB = g == c + 4 ? tkb + 8 * 24 : zero_s;
            const uint32_t mkb = mtable_s + ((kb - kb_base) * 48 + 2 * c) * 4;
            bool ok = !*reinterpret_cast<volatile int*>(&s_failed);
            if (ok && !mbar_wait(full_bar(s), phase)) {
              ok = false;
              s_failed = 1;
              report_error(a.err, kErrWaitFull);
            }
            if (!__any_sync(0xffffffffu, !ok)) {
              const uint32_t ag = ring_s + s * a.slot_bytes + off_g;
              const uint32_t ah = ring_s + s * a.slot_bytes + off_h;
              const float dg = u0 * h2f(lds_u16(ag + 208)), dh = u0 * h2f(lds_u16(ah + 208));
#pragma unroll 1
              for (uint32_t hf = 0; hf < 2; ++hf) {
                uint32_t L[2][4], Q[2][4];
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                  const uint32_t base = r ? ah : ag;
                  lds16_class<F>(base + 64 * hf + 16 * c, L[r]);
                  lds16_class<F>(base + 128 + 32 * hf + 16 * (c & 1), Q[r]);
                }
                q6i8_half(hf, L, Q, ag, ah, c, mkb, bA, bB, k16, k28, sHi, dg, dh, yacc);
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar(s));
            if (++s == a.ring) {
              s = 0;
              phase ^= 1;
            }
          }
          band_end(band, bi);
        }
      };
      const uint32_t kt_a = PART == 2 ? a.xpart : kt_lo, kt_z = PART == 1 ? a.xpart : kt_hi;
      const uint32_t kb_base = PART == 2 ? a.xpart * kq : 0u;
      switch (residue_class(fkb * kBlk)) {
        case 16: tmap_loop(std::integral_constant<int, 16>(), kt_a, kt_z, kb_base); break;
        case 8: tmap_loop(std::integral_constant<int, 8>(), kt_a, kt_z, kb_base); break;
        case 4: tmap_loop(std::integral_constant<int, 4>(), kt_a, kt_z, kb_base); break;
        case 2: tmap_loop(std::integral_constant<int, 2>(), kt_a, kt_z, kb_base); break;
        default: tmap_loop(std::integral_constant<int, 6>(), kt_a, kt_z, kb_base); break;
      }
      return;
    }
  }
  if constexpr (QT == 6 && I8) {
    if (a.fixed_blocks && !a.tmap_mode) {  // (tensor-map tiles without their loop take turns)
      const uint32_t fkb = warp;
      auto fixed_loop = [&](auto cls) {
        constexpr int F = decltype(cls)::value;
        const uint32_t kb = fkb;
        const float u0 = ublk_at(kb);
        const uint32_t tkb = table_s + (kb * 32 + 2 * c) * 24;
        const uint32_t bA = g == c ? tkb : zero_s;
        const uint32_t bB = g == c + 4 ? tkb + 8 * 24 : zero_s;
        const uint32_t mkb = mtable_s + (kb * 48 + 2 * c) * 4;
        const uint32_t off_g = pg_rb + kb * kBlk, off_h = ph_rb + kb * kBlk;
        uint32_t bi = 0;
        for (uint32_t band = 0; band < nbands; ++band) {
          bool ok = !*reinterpret_cast<volatile int*>(&s_failed);
          if (ok && !mbar_wait(full_bar(s), phase)) {
            ok = false;
            s_failed = 1;
            report_error(a.err, kErrWaitFull);
          }
          if (!__any_sync(0xffffffffu, !ok)) {
            const uint32_t ag = ring_s + s * a.slot_bytes + off_g;
            const uint32_t ah = ring_s + s * a.slot_bytes + off_h;
            const float dg = u0 * h2f(lds_u16(ag + 208)), dh = u0 * h2f(lds_u16(ah + 208));
#pragma unroll 1
            for (uint32_t hf = 0; hf < 2; ++hf) {
              uint32_t L[2][4], Q[2][4];
#pragma unroll
              for (int r = 0; r < 2; ++r) {
                const uint32_t base = r ? ah : ag;
                lds16_class<F>(base + 64 * hf + 16 * c, L[r]);
                lds16_class<F>(base + 128 + 32 * hf + 16 * (c & 1), Q[r]);
              }
              q6i8_half(hf, L, Q, ag, ah, c, mkb, bA, bB, k16, k28, sHi, dg, dh, yacc);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(empty_bar(s));
          if (++s == a.ring) {
            s = 0;
            phase ^= 1;
          }
          band_end(band, bi);
        }
      };
      switch (residue_class(fkb * kBlk)) {
        case 16: fixed_loop(std::integral_constant<int, 16>()); break;
        case 8: fixed_loop(std::integral_constant<int, 8>()); break;
        case 4: fixed_loop(std::integral_constant<int, 4>()); break;
        case 2: fixed_loop(std::integral_constant<int, 2>()); break;
        default: fixed_loop(std::integral_constant<int, 6>()); break;
      }
      return;
    }
  }
  // The same for Q4_K (144-byte blocks: every block starts on a 16-byte boundary, one loop):
  // the block's table addresses, scale of x and (integer path) sums of x are warp constants.
  if constexpr ((QT == 4 || QT == 5) && I8 && TXS == 0) {
    if (a.fixed_blocks && a.tmap_mode) {
      // Tensor-map tiles of K-tiled rows: warp w takes block w of every K-tile (all K-tiles have
      // the same width); the row offsets are the same in every tile, the block's x constants
      // (table addresses, scale, sums) change with the K-tile.
      const uint32_t off_g = pg_rb + warp * kBlk, off_h = ph_rb + warp * kBlk;
      uint32_t kt_lo, kt_hi;
      cta_ktiles(nkt, a.ksplit, kt_lo, kt_hi);
      uint32_t bi = 0;
      for (uint32_t band = 0; band < nbands; ++band) {
        for (uint32_t kt = kt_lo; kt < kt_hi; ++kt) {
          const uint32_t kb = kt * kq + warp;
          const float u0 = ublk_at(kb);
          const uint32_t tc = table_s + (kb * 32 + 8 * c) * 24;
          const uint32_t b0 = g == 2 * c ? tc : zero_s;
          const uint32_t b1 = g == 2 * c + 1 ? tc + 4 * 24 : zero_s;
          const uint2 xs = lds_v2(mtable_s + (kb * 8 + 2 * c) * 4);
          const float2 X = make_float2(__uint_as_float(xs.x), __uint_as_float(xs.y));
          bool ok = !*reinterpret_cast<volatile int*>(&s_failed);
          if (ok && !mbar_wait(full_bar(s), phase)) {
            ok = false;
            s_failed = 1;
            report_error(a.err, kErrWaitFull);
          }
          if (!__any_sync(0xffffffffu, !ok)) {
            const uint32_t slot = ring_s + s * a.slot_bytes;
            q4i8_block<QT == 5>(slot + off_g, slot + off_h, c, b0, b1, k28, sel_sc, m_lo, m_hi, sh_m, X, u0,
                                yacc);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(empty_bar(s));
          if (++s == a.ring) {
            s = 0;
            phase ^= 1;
          }
        }
        band_end(band, bi);
      }
      return;
    }
  }
  if constexpr (QT == 4 || QT == 5) {
    if (a.fixed_blocks && !a.tmap_mode) {
      const uint32_t kb = warp;
      float u0, u1 = 0.f;
      uint32_t b0 = 0, b1 = 0, tab_t[NT], bm_at[NT];
      float2 X = make_float2(0.f, 0.f);
      if constexpr (I8) {
        u0 = ublk_at(kb);
        const uint32_t tc = table_s + (kb * 32 + 8 * c) * 24;
        b0 = g == 2 * c ? tc : zero_s;
        b1 = g == 2 * c + 1 ? tc + 4 * 24 : zero_s;
        {
          const uint2 xs = lds_v2(mtable_s + (kb * 8 + 2 * c) * 4);
          X = make_float2(__uint_as_float(xs.x), __uint_as_float(xs.y));
        }
      } else {
        q4f16_consts(kb, tab_t, bm_at, u0, u1);
      }
      const uint32_t off_g = pg_rb + kb * kBlk, off_h = ph_rb + kb * kBlk;
      uint32_t bi = 0;
      for (uint32_t band = 0; band < nbands; ++band) {
        bool ok = !*reinterpret_cast<volatile int*>(&s_failed);
        if (ok && !mbar_wait(full_bar(s), phase)) {
          ok = false;
          s_failed = 1;
          report_error(a.err, kErrWaitFull);
        }
        if (!__any_sync(0xffffffffu, !ok)) {
          const uint32_t slot = ring_s + s * a.slot_bytes;
          if constexpr (I8)
            q4i8_block<QT == 5>(slot + off_g, slot + off_h, c, b0, b1, k28, sel_sc, m_lo, m_hi, sh_m, X, u0,
                       yacc);
          else
            q4f16_block(slot + off_g, slot + off_h, tab_t, bm_at, u0, u1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(s));
        if (++s == a.ring) {
          s = 0;
          phase ^= 1;
        }
        band_end(band, bi);
      }
      return;
    }
  }

  // Unit j (super-block kc0 + j) of a tile goes to warp (rot + j) mod nw, rot advancing by the
  // tile's super-block count, so the warps take turns when there are more warps than blocks.
  uint32_t bi = 0, rot = 0;
  uint32_t kt_lo, kt_hi;
  cta_ktiles(nkt, a.ksplit, kt_lo, kt_hi);
  for (uint32_t band = 0; band < nbands; ++band) {
  const uint32_t r0 = r_begin + band * kTileRows;
  uint32_t kc0 = kt_lo * kq + min(kt_lo, kr);
  for (uint32_t kt = kt_lo; kt < kt_hi; ++kt) {
    const uint32_t kc1 = kc0 + kq + (kt < kr ? 1u : 0u);
    bool ok = !*reinterpret_cast<volatile int*>(&s_failed);
    if (ok && !mbar_wait(full_bar(s), phase)) {
      ok = false;
      s_failed = 1;
      report_error(a.err, kErrWaitFull);
    }
    // warp-uniform, so that every lane takes the same path to the (.aligned) MMAs
    const bool failed = __any_sync(0xffffffffu, !ok);
    const uint32_t j = warp >= rot ? warp - rot : warp + nw - rot;
    const uint32_t kb = kc0 + j;
    const uint32_t slot = ring_s + s * a.slot_bytes;
    if (kb < kc1 && !failed) {
      // shared-memory addresses of this block in rows g and g+8 of the tile
      uint32_t ag, ah;
      if (a.seg_bytes == 0 || a.tmap_mode) {
        // whole rows back to back from the tile's aligned start (tensor-map slots: rows on
        // 16-byte boundaries, from the slot's start)
        const uint32_t delta = a.tmap_mode ? 0u : (r0 * rb32) & 15u;
        ag = slot + delta + pg_rb + j * kBlk;
        ah = slot + delta + ph_rb + j * kBlk;
      } else {
        const uint32_t off = kc0 * kBlk;
        ag = slot + pg * a.seg_bytes + (((r0 + pg) * rb32 + off) & 15u) + j * kBlk;
        ah = slot + ph * a.seg_bytes + (((r0 + ph) * rb32 + off) & 15u) + j * kBlk;
      }
      // the offset within 16 bytes that every lane's block shares, or 16 when they differ
      const uint32_t o16 = rows16 ? ((kb * kBlk) & 15u) : 16u;

      if constexpr (I8) {
        // Integer MMAs (batch 1). Column n of the MMA is sub-block n; the A registers of a step
        // hold 4 + 4 quants of one sub-block (8 consecutive elements of it per thread), B the
        // three limbs of the same 8 elements of x, read by the 4 lanes of the column's group.
        const float u0 = ublk_at(kb);
        if constexpr (QT == 4 || QT == 5) {
          const uint32_t tc = table_s + (kb * 32 + 8 * c) * 24;
          const uint32_t b0 = g == 2 * c ? tc : zero_s;
          const uint32_t b1 = g == 2 * c + 1 ? tc + 4 * 24 : zero_s;
          const uint2 xs = lds_v2(mtable_s + (kb * 8 + 2 * c) * 4);
          const float2 X = make_float2(__uint_as_float(xs.x), __uint_as_float(xs.y));
          q4i8_block<QT == 5>(ag, ah, c, b0, b1, k28, sel_sc, m_lo, m_hi, sh_m, X, u0, yacc);
        } else {
          // Q6_K: per half, 4 steps: s < 2 the low-nibble group (sub-block c, words 2(s&1),
          // 2(s&1)+1 of the thread's 16 ql bytes), s >= 2 the high-nibble group (sub-block c+4)
          const float dg = u0 * h2f(lds_u16(ag + 208)), dh = u0 * h2f(lds_u16(ah + 208));
          const uint32_t o0 = o16 & 15u;
          const bool same = o16 < 16u;
          const uint32_t fs = 8 * (o0 & 3);
          // B fragments: thread (g, c) reads the table in steps 0-1 when g == c and in steps 2-3
          // when g == c + 4 (entries kb*32 + 16 hf + 8 (st >> 1) + 2c + (st & 1), 24 bytes each),
          // else the zero region; every step's address is one of two bases plus a constant.
          const uint32_t tkb = table_s + (kb * 32 + 2 * c) * 24;
          const uint32_t bA = g == c ? tkb : zero_s;
          const uint32_t bB = g == c + 4 ? tkb + 8 * 24 : zero_s;
          // accumulator start values: entries ((kb * 2 + hf) * 3 + l) * 8 + 2c, 4 bytes each
          const uint32_t mkb = mtable_s + (kb * 48 + 2 * c) * 4;
          auto half = [&](uint32_t hf, const uint32_t (&L)[2][4], const uint32_t (&Q)[2][4]) {
            q6i8_half(hf, L, Q, ag, ah, c, mkb, bA, bB, k16, k28, sHi, dg, dh, yacc);
          };
#pragma unroll 1
          for (uint32_t hf = 0; hf < 2; ++hf) {
            uint32_t L[2][4], Q[2][4];
            if (!same)
              q6_load_half<-2>(ag, ah, c, hf, 0, L, Q);
            else if (o0 == 0)
              q6_load_half<-1>(ag, ah, c, hf, fs, L, Q);
            else if (o0 == 8)
              q6_load_half<8>(ag, ah, c, hf, fs, L, Q);
            else if ((o0 & 3u) == 0)
              q6_load_half<4>(ag, ah, c, hf, fs, L, Q);
            else if (o0 < 4)
              q6_load_half<0>(ag, ah, c, hf, fs, L, Q);
            else if (o0 < 8)
              q6_load_half<1>(ag, ah, c, hf, fs, L, Q);
            else if (o0 < 12)
              q6_load_half<2>(ag, ah, c, hf, fs, L, Q);
            else
              q6_load_half<3>(ag, ah, c, hf, fs, L, Q);
            half(hf, L, Q);
          }
        }
      } else if constexpr (QT == 4) {
        uint32_t tab_t[NT], bm_at[NT];
        float u0, u1;
        q4f16_consts(kb, tab_t, bm_at, u0, u1);
        q4f16_block(ag, ah, tab_t, bm_at, u0, u1);
      } else {
        // Q6_K, batch 1: thread (g, c) owns sub-blocks c and c+4 of each half of the block
        const float u0 = ublk_at(kb);
        const float dg = u0 * h2f(lds_u16(ag + 208)), dh = u0 * h2f(lds_u16(ah + 208));
        const uint32_t tab_kb = tab_on ? table_s + kb * 1024 + tab_lane : zero_s;
        // the block's quants, loaded in the form the rows' common alignment allows
        uint32_t L[2][2][4], Q[2][2][4];
        const uint32_t o0 = o16 & 15u;
        if (o16 < 16u) {
          const uint32_t fs = 8 * (o0 & 3);
          switch (o0 >> 2) {
            case 0:
              if (o0 == 0) q6_load<-1>(ag, ah, c, fs, L, Q);
              else q6_load<0>(ag, ah, c, fs, L, Q);
              break;
            case 1: q6_load<1>(ag, ah, c, fs, L, Q); break;
            case 2: q6_load<2>(ag, ah, c, fs, L, Q); break;
            default: q6_load<3>(ag, ah, c, fs, L, Q); break;
          }
        } else {
          q6_load<-2>(ag, ah, c, 0, L, Q);
        }
        q6_block(ag, ah, c, tab_kb, k24, kT, kT13, dg, dh, L, Q, yacc);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar(s));
    if (++s == a.ring) {
      s = 0;
      phase ^= 1;
    }
    rot += kc1 - kc0;
    if (rot >= nw) rot -= nw;
    kc0 = kc1;
  }  // K-tiles of the band

  band_end(band, bi);
  }  // bands
}

// ---------------------------------------------------------------- the kernels

// QT: 4, 5 or 6. NT: n8 tiles per MMA step (2 when batch 5..8 takes hi and lo in separate tiles).
// HILO: x enters as hi + lo (else hi only). I8 (batch 1): integer MMAs, A = the raw quants as
// bytes, x as three signed byte limbs (24-bit fixed point per 256-element block), the eight MMA
// columns separating sub-blocks.
template <int QT, int NT, bool HILO, bool I8, bool XP = false>
__global__ void __launch_bounds__((kMaxWarps + 1) * 32, 1) warpmma_kernel(const __grid_constant__ WarpMmaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ WarpMmaShared sh;
  uint8_t* base = smem_base(smem);
  init_ring(a, base, sh);
  pdl_launch_dependents();
  uint32_t s = 0, phase = 0;
  const JobArgs v = job_of(a);
  if ((threadIdx.x >> 5) == a.nw) {
    if (!(a.flags & KQ_FLAG_WEIGHTS_STATIC)) pdl_wait();
    uint32_t issued = 0;
    produce_job<QT, XP>(a, v, base, sh, s, phase, issued);
    return;
  }
  pdl_wait();  // x may be the previous kernel's output
  if constexpr (XP) {
    // x in two parts: the first part's table and K-tiles, then the second's (the ring position
    // and the partial rows in shared memory carry over)
    consume_job<QT, NT, HILO, I8, 0, 1>(a, v, nullptr, base, sh, s, phase);
    consume_job<QT, NT, HILO, I8, 0, 2>(a, v, nullptr, base, sh, s, phase);
  } else {
    consume_job<QT, NT, HILO, I8>(a, v, nullptr, base, sh, s, phase);
  }
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Adds n to *cnt with release semantics: every store this CTA made before (ordered by the barrier
// its consumers met first) is visible, at the scope, before the count is.
__device__ __forceinline__ void red_release_gpu(unsigned long long* cnt, uint32_t n) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(cnt), "l"(static_cast<unsigned long long>(n))
               : "memory");
}
__device__ __forceinline__ void red_release_sys(unsigned long long* cnt, uint32_t n) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(cnt), "l"(static_cast<unsigned long long>(n))
               : "memory");
}

// Bounded wait (acquire; system scope when other GPUs add to the counter, else GPU scope) by one
// thread until *cnt >= target; on giving up it records kErrWaitPeer and returns false (at once
// when the CTA or an earlier wait already failed).
__device__ __forceinline__ bool wait_at_least(unsigned* err, const unsigned long long* cnt,
                                              unsigned long long target, bool sys, const int* failed) {
  auto load = [&]() { return sys ? ld_acquire_sys(cnt) : ld_acquire_gpu(cnt); };
  if (load() >= target) return true;
  if (*reinterpret_cast<const volatile int*>(failed) || (err && *reinterpret_cast<volatile unsigned*>(err)))
    return false;
  const uint64_t t0 = globaltimer();
  while (load() < target) {
    if (globaltimer() - t0 > kWaitBudgetNs) {
      report_error(err, kErrWaitPeer);
      return false;
    }
  }
  return true;
}

// A lone batch-1 integer matvec that also does a row-sharded stack's exchange. Counted form
// (TX false, q.y.tagged 0): before its consumers read x (a full vector other GPUs push into), one
// thread waits (bounded, acquire, system scope) until this rank's counter for x reaches this
// step's target; its flushes store the outputs below push_rows into every rank's full vector; once
// they are stored, the CTA adds their count to every rank's counter (release, system scope).
// Tagged form (q.y.tagged 1; TX: x is tagged too): the outputs go out as 8-byte (value, tag)
// stores and x's elements are each waited for until they carry this step's tag, so there is no
// fence, no counter and no round trip on the critical path. The producer streams the weights from
// the start, the wait overlapping the first tiles' copies.
template <int QT, int TXS, bool XP = false>
__global__ void __launch_bounds__((kMaxWarps + 1) * 32, 1)
    warpmma_push_kernel(const __grid_constant__ WarpMmaArgs a, const __grid_constant__ PushArgs q) {
  constexpr bool TX = TXS > 0;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ WarpMmaShared sh;
  uint8_t* base = smem_base(smem);
  init_ring(a, base, sh);
  pdl_launch_dependents();
  uint32_t s = 0, phase = 0;
  const JobArgs v = job_of(a);
  if ((threadIdx.x >> 5) == a.nw) {
    if (!(a.flags & KQ_FLAG_WEIGHTS_STATIC)) pdl_wait();
    uint32_t issued = 0;
    produce_job<QT, XP>(a, v, base, sh, s, phase, issued);
    return;
  }
  pdl_wait();
  const uint32_t nthr = a.nw * 32;
  if (threadIdx.x == 0) {
    if (q.y.tagged || TX) {
      const unsigned long long e = ld_epoch(q.epoch) - 1ull;
      sh.tag_x = static_cast<uint32_t>(e * q.wait_mul + q.wait_add);
      sh.tag_out = static_cast<uint32_t>(e * q.push_mul + q.push_add);
      sh.x_slots = q.x_slots;
    }
    if (!TX && q.y.wait_cnt) {
      const unsigned long long target = (ld_epoch(q.epoch) - 1ull) * q.wait_mul + q.wait_add;
      if (!wait_at_least(a.err, q.y.wait_cnt, target, true, &sh.failed)) sh.failed = 1;
    }
  }
  named_barrier(1, nthr);
  if constexpr (XP) {
    consume_job<QT, 1, false, true, TXS, 1>(a, v, &q.y, base, sh, s, phase);
    consume_job<QT, 1, false, true, TXS, 2>(a, v, &q.y, base, sh, s, phase);
  } else {
    consume_job<QT, 1, false, true, TXS>(a, v, &q.y, base, sh, s, phase);
  }
  if (q.y.tagged) return;  // no counts
  named_barrier(1, nthr);  // every consumer's outputs are stored
  if (threadIdx.x == 0 && q.y.npush) {
    uint32_t r_begin, r_end;
    cta_rows(v, a.ksplit, r_begin, r_end);
    const uint32_t o0 = r_begin / v.row_unit, o1 = r_end / v.row_unit, pr = q.y.push_rows;
    const uint32_t pushed = o1 > pr ? (o0 < pr ? pr - o0 : 0u) : o1 - o0;
    for (uint32_t rk = 0; rk < q.y.npush; ++rk) red_release_sys(q.y.counter[rk], pushed);
  }
}

// dst[i] = the value of tagged element i of src once it carries the tag (bounded waits).
__global__ void tagged_unpack_kernel(float* dst, const unsigned long long* src, uint64_t n,
                                     const unsigned long long* epoch, uint64_t mul, uint64_t add,
                                     unsigned* err) {
  const uint32_t want = static_cast<uint32_t>((ld_epoch(epoch) - 1ull) * mul + add);
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
    unsigned long long w = ld_tagged(src + i);
    if (static_cast<uint32_t>(w >> 32) != want) {
      const uint64_t t0 = globaltimer();
      while (static_cast<uint32_t>(w >> 32) != want) {
        if ((err && *reinterpret_cast<volatile unsigned*>(err)) || globaltimer() - t0 > kWaitBudgetNs) {
          report_error(err, kErrWaitPeer);
          break;
        }
        w = ld_tagged(src + i);
      }
    }
    dst[i] = __uint_as_float(static_cast<uint32_t>(w));
  }
}

// A chain: the batch-1 integer matvecs p.job[0..njobs) of one type and k in one launch, each
// reading the previous one's output. The producer streams the jobs' tiles back to back, so the
// next matrix's weights are in flight while the consumers finish a matrix and wait for its
// output. Between jobs, instead of a kernel boundary: every CTA, once its outputs of job j are
// stored (on this GPU, and with a push on every rank's), adds its output count to job j's
// counter(s) (release; system scope when pushing to other GPUs); job j + 1's consumers wait
// (bounded, acquire) until their counter reaches *epoch * wait_target, i.e. until every CTA of
// every rank has stored its part of x for this token. The counters only grow: *epoch, which the
// caller advances once per token, makes each token's targets its own. All CTAs of the grid wait
// on one another, so the grid is one CTA per SM and the CTAs must all be resident: nothing else
// may hold an SM for good while a chain runs (kernels before it in the stream finish on their
// own; kernels after it start only as its CTAs exit).
template <int QT>
__global__ void __launch_bounds__((kMaxWarps + 1) * 32, 1)
    warpmma_chain_kernel(const __grid_constant__ ChainParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ WarpMmaShared sh;
  uint8_t* base = smem_base(smem);
  // the layout (ring, tiles, shared-memory regions) is the same for every job: its fields are read
  // at fixed parameter offsets, as a lone launch reads them; only each job's own fields vary
  const WarpMmaArgs& a = p.lay;
  init_ring(a, base, sh);
  pdl_launch_dependents();
  const uint32_t nw = a.nw, nthr = nw * 32;
  uint32_t s = 0, phase = 0;
  if ((threadIdx.x >> 5) == nw) {
    if (!(a.flags & KQ_FLAG_WEIGHTS_STATIC)) pdl_wait();
    uint32_t issued = 0;
    bool ok = true;
    for (uint32_t j = 0; j < p.njobs && ok; ++j) ok = produce_job<QT>(a, p.job[j], base, sh, s, phase, issued);
    if (!ok && (threadIdx.x & 31) == 0) {
      // a wait gave up: before the CTA ends, let the copies still in flight into its ring land
      // (each slot's last phase; bounded like every wait)
      const uint32_t n = min(issued, a.ring);
      uint64_t* bars = reinterpret_cast<uint64_t*>(base + a.bars_off);
      uint32_t ss = s, ph = phase;
      for (uint32_t i = 0; i < n; ++i) {
        if (ss == 0) {
          ss = a.ring;
          ph ^= 1;
        }
        --ss;
        mbar_wait_sleep(smem_u32(&bars[ss]), ph);
      }
    }
    return;
  }
  pdl_wait();  // the first job's x may be the previous kernel's output
  // The current job's own fields live in shared memory: the tile loops then hold no register for
  // them (they are read where used, at the prologue and the flushes), as a lone launch reads its
  // fields from the parameter bank.
  __shared__ JobArgs s_job;
  __shared__ ChainSync s_sync;
  __shared__ unsigned long long s_epoch;
  __shared__ uint32_t s_zero;
  if (threadIdx.x == 0) {
    s_epoch = p.sync[0].wait_cnt || p.njobs > 1 ? ld_epoch(p.epoch) : 0ull;
    s_zero = 0;
  }
  for (uint32_t j = 0; j < p.njobs; ++j) {
    // thread 0 has read the previous job's counters from s_sync for its signal before anyone
    // overwrites them
    if (j) named_barrier(1, nthr);
    // the job's fields into shared memory, a word per consumer thread
    static_assert(sizeof(JobArgs) % 4 == 0 && sizeof(ChainSync) % 4 == 0, "word copies");
    constexpr uint32_t kJobWords = sizeof(JobArgs) / 4, kSyncWords = sizeof(ChainSync) / 4;
    for (uint32_t i = threadIdx.x; i < kJobWords + kSyncWords; i += nthr) {
      if (i < kJobWords)
        reinterpret_cast<uint32_t*>(&s_job)[i] = reinterpret_cast<const uint32_t*>(&p.job[j])[i];
      else
        reinterpret_cast<uint32_t*>(&s_sync)[i - kJobWords] =
            reinterpret_cast<const uint32_t*>(&p.sync[j])[i - kJobWords];
    }
    if (threadIdx.x == 0) {
      // x is complete once the counter of the job that wrote it reaches this step's target
      const ChainSync& y = p.sync[j];
      if (y.wait_cnt && !wait_at_least(a.err, y.wait_cnt, s_epoch * y.wait_target, y.npush != 0, &sh.failed))
        sh.failed = 1;
    }
    named_barrier(1, nthr);
    consume_job<QT, 1, false, true>(a, s_job, &s_sync, base, sh, s, phase,
                                    *reinterpret_cast<volatile uint32_t*>(&s_zero));
    named_barrier(1, nthr);  // every consumer's outputs of job j are stored
    if (threadIdx.x == 0 && s_sync.counter[0]) {
      uint32_t r_begin, r_end;
      cta_rows(s_job, a.ksplit, r_begin, r_end);
      const uint32_t o0 = r_begin / s_job.row_unit, o1 = r_end / s_job.row_unit;
      const uint32_t pr = s_sync.push_rows;
      if (s_sync.npush) {
        const uint32_t pushed = o1 > pr ? (o0 < pr ? pr - o0 : 0u) : o1 - o0;
        for (uint32_t rk = 0; rk < s_sync.npush; ++rk) red_release_sys(s_sync.counter[rk], pushed);
      } else {
        red_release_gpu(s_sync.counter[0], o1 - o0);
      }
    }
  }
}

struct Variant {
  const void* fn;
  int qt, nt;
  bool hilo;
};

template <int QT, int NT, bool HILO, bool I8 = false, bool XP = false>
Variant variant() {
  return Variant{reinterpret_cast<const void*>(&warpmma_kernel<QT, NT, HILO, I8, XP>), QT, NT, HILO};
}

// (the last: the Q6_K integer kernel compiled for x in two parts, which a plan with xpart takes
// instead of mode 5's)
const Variant kVariants[] = {variant<4, 1, true>(), variant<4, 2, true>(), variant<4, 1, false>(),
                             variant<6, 1, false>(), variant<4, 1, false, true>(),
                             variant<6, 1, false, true>(), variant<5, 1, false, true>(),
                             variant<6, 1, false, true, true>()};
constexpr int kXPartVariant = 7;

// The push kernel of a type (Q4_K, Q5_K or Q6_K) for x plain (txs 0), tagged (1), or tagged
// with several split-K slots (2).
template <int TXS>
const void* push_fn_t(uint32_t type) {
  return type == KQ_TYPE_Q4_K   ? reinterpret_cast<const void*>(&warpmma_push_kernel<4, TXS>)
         : type == KQ_TYPE_Q5_K ? reinterpret_cast<const void*>(&warpmma_push_kernel<5, TXS>)
                                : reinterpret_cast<const void*>(&warpmma_push_kernel<6, TXS>);
}
// (xp: the Q6_K kernel compiled for x in two parts, plain x)
const void* push_fn(uint32_t type, int txs, bool xp = false) {
  if (xp && type == KQ_TYPE_Q6_K && txs == 0)
    return reinterpret_cast<const void*>(&warpmma_push_kernel<6, 0, true>);
  return txs == 0 ? push_fn_t<0>(type) : txs == 1 ? push_fn_t<1>(type) : push_fn_t<2>(type);
}

// The chain kernel of a type (Q4_K, Q5_K or Q6_K).
const void* chain_fn(uint32_t type) {
  return type == KQ_TYPE_Q4_K   ? reinterpret_cast<const void*>(&warpmma_chain_kernel<4>)
         : type == KQ_TYPE_Q5_K ? reinterpret_cast<const void*>(&warpmma_chain_kernel<5>)
                                : reinterpret_cast<const void*>(&warpmma_chain_kernel<6>);
}

}  // namespace wm

using namespace wm;

int warpmma_prepare(kq_ctx* ctx) {
  for (const Variant& v : kVariants) {
    const cudaError_t e =
        cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, ctx->max_smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute", "warp-MMA matvec kernel");
  }
  for (uint32_t t : {uint32_t(KQ_TYPE_Q4_K), uint32_t(KQ_TYPE_Q5_K), uint32_t(KQ_TYPE_Q6_K)}) {
    cudaError_t e =
        cudaFuncSetAttribute(chain_fn(t), cudaFuncAttributeMaxDynamicSharedMemorySize, ctx->max_smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute", "warp-MMA chain kernel");
    for (int txs : {0, 1, 2})
      for (bool xp : {false, true}) {
        e = cudaFuncSetAttribute(push_fn(t, txs, xp), cudaFuncAttributeMaxDynamicSharedMemorySize, ctx->max_smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute", "warp-MMA push kernel");
      }
  }
  return KQ_OK;
}

bool warpmma_supports(const kq_matvec_desc& d) {
  if (d.type == KQ_TYPE_Q4_K) return d.batch >= 1 && d.batch <= 8;
  if (d.type == KQ_TYPE_Q6_K || d.type == KQ_TYPE_Q5_K) return d.batch == 1;
  return false;
}

namespace {

// A planned warp-MMA launch: the kernel's arguments, the variant, and the launch shape.
struct WarpMmaPlan {
  WarpMmaArgs args;
  int mode;  // index into kVariants
  uint32_t smem, grid, block;
};

// Chooses the variant, the tiles and the shared-memory layout of one matvec (arguments already
// checked by the caller), as the standalone launch uses them.
int warpmma_plan(kq_ctx* ctx, const kq_matvec_desc& d, uint64_t ldx, uint64_t ldy, const char* call,
                 WarpMmaPlan& plan, uint32_t ksplit = 1, bool compact = true, bool tmap_fixed = true,
                 bool xparts = true) {
  const bool q4 = d.type == KQ_TYPE_Q4_K;
  const bool q5 = d.type == KQ_TYPE_Q5_K;  // Q4_K's layout plus qh: the Q4_K forms, integer only
  const bool q45 = q4 || q5;
  const uint32_t blk = q4 ? kQ4KBytes : q5 ? kQ5KBytes : kQ6KBytes;
  const uint32_t nb = d.k / kQK;
  const uint64_t rb = uint64_t(nb) * blk;
  // tile: 16 row segments of up to kc super-blocks (kc = the consumer warps), one bulk copy
  // each (the 16-byte-aligned superset, so up to 30 bytes more), at a pitch whose residue mod 128
  // makes the consumers' 16-byte loads free of bank conflicts: 16 for Q4_K (rows g, g+1
  // interleave their 32-byte strides), 64 for Q6_K (rows g, g+1 take the two halves of 128 B)
  const uint32_t target = q45 ? 16u : 64u;
  auto slot_for = [&](uint32_t kc, uint32_t& seg_out) {
    uint32_t seg_ = ((kc * blk + 30 + 15) / 16) * 16;
    while (seg_ % 128 != target) seg_ += 16;
    seg_out = seg_;
    return kTileRows * seg_;
  };
  uint32_t nkt = (nb + kTileBlocks - 1) / kTileBlocks;
  uint32_t nwc = (nb + nkt - 1) / nkt;
  uint32_t seg = 0;
  uint32_t slot = slot_for(nwc, seg);
  // A tile of whole rows goes in one copy (the copy engine's cost is per copy, ~75 ns per SM,
  // so many small copies cap the bandwidth), its rows back to back.
  // Rows on a pitch of 0 mod 128 would put a quarter-warp's two rows on the same banks: such a
  // tile goes in two copies, its rows 8..15 kSplitGap bytes further (see pg in the kernel).
  const bool split = rb % 128 == 0;
  auto whole_rows = [&]() {
    if (nkt != 1) return;
    seg = 0;
    slot = static_cast<uint32_t>(((uint64_t(kTileRows) * rb + 32 + (split ? kSplitGap : 0) + 127) / 128) * 128);
  };
  whole_rows();

  // mode: Q4_K hi+lo in one n-tile (batch <= 4), hi+lo in two (batch 5..8), or hi only when
  // the table of two would not leave room for a ring of two slots
  int mode;  // index into kVariants
  uint32_t ncol;
  uint64_t table_bytes, mtable_bytes;
  const uint32_t ublk_bytes = ((nb * d.batch * 4 + 15) / 16) * 16;
  const uint64_t fixed_min =
      2 * uint64_t(slot) + kTileRows * kMaxWarps * d.batch * 4 + ublk_bytes + kZeroBytes + 256 + 128;
  // batch 1: the integer kernel, whose table is x's three byte limbs (3 bytes per element) plus
  // per-sub-block sums (Q6_K: the MMAs' C init, Q4_K: the min term's sums of x)
  const uint64_t i8_table = uint64_t(nb) * kQK * 3;
  const uint64_t i8_mtable = q45 ? uint64_t(nb) * 8 * 4 : uint64_t(nb) * 2 * 3 * 8 * 4;
  const bool want_i8 = (d.flags & kFlagAltBatch1) == 0 || q5;
  if (d.batch == 1 && want_i8 &&
      i8_table + i8_mtable + fixed_min <= uint64_t(ctx->max_smem)) {
    mode = q4 ? 4 : q5 ? 6 : 5, ncol = 8;
    table_bytes = i8_table;
    mtable_bytes = i8_mtable;
  } else if (q5) {
    return fail(KQ_E_UNSUPPORTED, call,
                "k " + std::to_string(d.k) + " does not fit the Q5_K warp-MMA kernel's shared memory");
  } else if (q4) {
    auto sizes = [&](uint32_t nt_, uint32_t ncol_) {
      table_bytes = uint64_t(nb) * nt_ * ncol_ * kNStride;
      mtable_bytes = uint64_t(nb) * nt_ * ncol_ * 16;
      return table_bytes + mtable_bytes;
    };
    if (d.batch <= 4 && sizes(1, 2 * d.batch) + fixed_min <= uint64_t(ctx->max_smem)) {
      mode = 0, ncol = 2 * d.batch;
    } else if (d.batch > 4 && sizes(2, d.batch) + fixed_min <= uint64_t(ctx->max_smem)) {
      mode = 1, ncol = d.batch;
    } else {
      mode = 2, ncol = d.batch;
      sizes(1, d.batch);
    }
  } else {
    mode = 3, ncol = 8;
    table_bytes = uint64_t(nb) * 1024;
    mtable_bytes = 0;
  }
  // Narrower K-tiles (fewer consumer warps, smaller slots) until two slots and one band of
  // partial rows fit beside the table.
  auto need_for = [&](uint32_t slot_) {
    return table_bytes + mtable_bytes + ublk_bytes + kZeroBytes + 16 + 2 * 8 * 8 + 128 +
           2 * uint64_t(slot_) + uint64_t(kTileRows) * kMaxWarps * d.batch * 4;
  };
  while (need_for(slot) > uint64_t(ctx->max_smem) && nwc > 1) {
    ++nkt;
    nwc = (nb + nkt - 1) / nkt;
    slot = slot_for(nwc, seg);
  }
  // Consumer warps: kMaxWarps (the warps taking turns over a tile's blocks), or one per block of
  // the widest K-tile. Measured on B200: a warp fixed to one block of whole-row tiles on 16-byte
  // boundaries runs the integer path's fixed-block loop (every per-block constant hoisted; for
  // Q6_K one load form per block alignment): 7% faster than turns for Q4_K, 3% for Q6_K. Else
  // turns are 3% faster for Q4_K up to batch 4 (more warps hide more latency), 2% slower at
  // batch 8 (the two-tile MMAs' registers).
  const bool rows16 = rb % 16 == 0;
  const bool fixed_ok = (q45 || mode == 5) && nkt == 1 && seg == 0 && rows16;
  const bool turns = fixed_ok ? false : q45 ? d.batch <= 4 : !rows16;
  const bool per_block = !turns != ((d.flags & kFlagWarpPerBlock) != 0);
  uint32_t nw = per_block ? nwc : kMaxWarps;
  const uint32_t rb128 = static_cast<uint32_t>(rb % 128);
  const uint32_t row_perm = (seg == 0 && (rb128 == 32 || rb128 == 96)) ? 1u : 0u;
  if (need_for(slot) > uint64_t(ctx->max_smem))
    return fail(KQ_E_UNSUPPORTED, call,
                "k " + std::to_string(d.k) + " with batch " + std::to_string(d.batch) +
                    " does not fit the warp-MMA kernel's shared memory");
  // A CTA with fewer rows than a tile's 16 (short matrices, row shards): its slots hold only the
  // rows it has, so that more slots, and more tiles in flight, fit beside the table. The
  // consumers still read 16 rows of a slot; the rows it lacks lie past it, in the next slot or,
  // from the last slot, in the table that follows the ring, and feed outputs nobody stores.
  // (Segmented tiles only, whose rows each have their own copy; chains keep full slots, so that
  // every job of a launch has one layout.)
  //
  // K-tiled rows (segmented tiles) of a CTA with a whole band (Q4_K, Q5_K: three whole bands; with
  // fewer, measured slower: 70B 2-way q|k|v 12.6 -> 13.7 us, o 9.9 -> 10.6 us, while the Q6_K
  // down projection gained at any band count, 2-way 39.1 -> 35.5 us): the whole bands come in
  // by a 3-D tensor map, one TMA copy per tile (two for a split tile) instead of one bulk copy
  // per row, whose per-copy cost capped the producer (measured on B200: one copy per tile made
  // the 70B gate|up 20% faster). It needs equal K-tiles, rows and K-tiles on 16-byte boundaries
  // (Q6_K: K-tiles of whole 8-block groups, 1680 bytes) and a row pitch the consumers' loads
  // take without bank conflicts (the box lands in one piece, its rows back to back, so that its
  // shared-memory start stays on 128 bytes): Q4_K and Q5_K rows 16 mod 32 bytes apart, the box
  // one block wider than the K-tile when the K-tile alone is 0 mod 128 (the extra block is the
  // next K-tile's first, read again from L2, or past the row's end, filled with zeros); Q6_K rows
  // 64 mod 128 apart, or 32 / 96 with MMA rows paired two apart, as for whole-row tiles.
  const uint32_t ru = d.epilogue != KQ_EPILOGUE_NONE ? 2 : 1;
  const uint64_t units = d.rows / ru;
  const uint64_t groups =
      std::max<uint64_t>(1, std::min<uint64_t>(ctx->sm_count / std::max<uint32_t>(ksplit, 1), units));
  const uint64_t rpc = (units + groups - 1) / groups * ru;  // rows of the fullest CTA
  bool tmap = false, tperm = false;
  uint32_t kbox = nwc;            // blocks in a box row
  uint32_t tp = nwc * blk;        // the tensor-map layout's row pitch
  if (compact && seg != 0 && rpc >= (q45 ? 3u : 1u) * kTileRows && nb % nkt == 0 && rb % 16 == 0 &&
      (q45 || (nb % 8 == 0 && nwc % 8 == 0))) {
    if (q45) {
      if (tp % 32 != 16) kbox = nwc + 1, tp = kbox * blk;
      tmap = tp % 32 == 16;
    } else {
      const uint32_t res = tp % 128;
      tperm = res == 32 || res == 96;
      tmap = tperm || res == 64;
    }
  }
  CUtensorMap tm_map;
  if (tmap) {
    std::memset(&tm_map, 0, sizeof(tm_map));
    int erc;
    if (q45) {
      const uint64_t dims[3] = {blk, nb, d.rows}, strides[2] = {blk, rb};
      const uint32_t box[3] = {blk, kbox, kTileRows};
      erc = encode_tensor_map(&tm_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, reinterpret_cast<const void*>(d.w),
                              dims, strides, box, call);
    } else {
      const uint64_t dims[3] = {kQ6KBytes, nb / 8, d.rows}, strides[2] = {8 * kQ6KBytes, rb};
      const uint32_t box[3] = {kQ6KBytes, nwc / 8, kTileRows};  // 8 blocks = 210 8-byte words
      erc = encode_tensor_map(&tm_map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, reinterpret_cast<const void*>(d.w),
                              dims, strides, box, call);
    }
    if (erc) return erc;
    seg = tp;
    slot = static_cast<uint32_t>(((uint64_t(kTileRows) * tp + 127) / 128) * 128);
    // Q4_K / Q5_K at batch 1: warp w fixed to block w of every K-tile, as for whole-row tiles
    if (tmap_fixed && (mode == 4 || mode == 5 || mode == 6) && !(d.flags & kFlagWarpPerBlock)) nw = nwc;
  } else if (compact && seg != 0) {
    const uint32_t cslot = static_cast<uint32_t>(((rpc * seg + 127) / 128) * 128);
    if (rpc < kTileRows && kTileRows * seg - cslot <= table_bytes + mtable_bytes) slot = cslot;
  }
  // partial rows of up to 16 bands between flushes, in what two ring slots leave
  const uint32_t band_red = kTileRows * nw * d.batch * 4;
  auto ring_for = [&](uint64_t table, uint32_t bands) {
    const uint64_t tail_ = table + ublk_bytes + kZeroBytes + 16 + uint64_t(bands) * band_red + 2 * 8 * 8 + 128;
    return tail_ < uint64_t(ctx->max_smem) ? (uint64_t(ctx->max_smem) - tail_) / slot : 0;
  };
  // x in two parts (Q6_K tensor-map tiles of a lone launch or a push of a plain x, warp w on
  // block w, no prologue or epilogue): when the whole x table (3.75 bytes an element: K = 28672
  // takes 105 KB) leaves room for only two ring slots, the table holds the first half of the
  // K-tiles, then the second's (each warp rebuilds its own entries once every band has had its
  // first part); every band's partial rows stay in shared memory in between. A third slot of
  // 54 KB keeps more of the CTA's weights in flight.
  uint32_t xpart = 0;
  const uint32_t cta_bands = static_cast<uint32_t>((rpc + kTileRows - 1) / kTileRows);
  if (xparts && tmap && mode == 5 && nw == nwc && tmap_fixed && !(d.flags & kFlagWarpPerBlock) && ksplit <= 1 &&
      d.prologue == KQ_PROLOGUE_NONE && d.epilogue == KQ_EPILOGUE_NONE && nkt >= 2 &&
      cta_bands <= 16 && ring_for(table_bytes + mtable_bytes, 16) < 3) {
    const uint32_t kh = (nkt + 1) / 2, nbh = kh * (nb / nkt);
    const uint64_t tb = uint64_t(nbh) * kQK * 3, mb = uint64_t(nbh) * 2 * 3 * 8 * 4;
    if (ring_for(tb + mb, cta_bands) >= 3) {
      xpart = kh;
      table_bytes = tb;
      mtable_bytes = mb;
    }
  }
  const uint64_t base_need = need_for(slot) - uint64_t(kTileRows) * kMaxWarps * d.batch * 4;
  const uint32_t fb = xpart ? cta_bands
                            : static_cast<uint32_t>(std::min<uint64_t>(
                                  16, std::min<uint64_t>(kRedBudget, uint64_t(ctx->max_smem) - base_need) / band_red));
  const uint32_t red_bytes = fb * band_red;
  const uint64_t tail =
      table_bytes + mtable_bytes + ublk_bytes + kZeroBytes + 16 + red_bytes + 2 * 8 * 8 + 128;
  uint32_t ring = std::min<uint64_t>(8, (uint64_t(ctx->max_smem) - tail) / slot);
  ring = std::max<uint32_t>(2, ring);

  WarpMmaArgs args;
  args.W = reinterpret_cast<const uint8_t*>(d.w);
  args.x = reinterpret_cast<const float*>(d.x);
  args.y = reinterpret_cast<float*>(d.y);
  args.err = ctx->err;
  args.ldx = ldx;
  args.ldy = ldy;
  args.total_bytes = uint64_t(d.rows) * rb;
  args.row_bytes = rb;
  args.rows = d.rows;
  args.nb = nb;
  args.batch = d.batch;
  args.nkt = nkt;
  args.nw = nw;
  args.ring = ring;
  args.slot_bytes = slot;
  args.seg_bytes = seg;
  args.table_off = ring * slot;
  args.mtable_off = static_cast<uint32_t>(args.table_off + table_bytes);
  args.ublk_off = static_cast<uint32_t>(((args.mtable_off + mtable_bytes + 15) / 16) * 16);
  args.zero_off = args.ublk_off + ublk_bytes;
  args.red_off = args.zero_off + kZeroBytes;
  args.zero = 0;
  args.row_perm = tmap ? (tperm ? 1u : 0u) : row_perm;
  args.split_tile = tmap ? 0u : (seg == 0 && split) ? 1u : 0u;
  args.tmap_mode = tmap ? 1u : 0u;
  args.tile_pitch = tmap ? tp : 0u;
  args.xpart = xpart;
  if (tmap) args.tmap = tm_map;
  else std::memset(&args.tmap, 0, sizeof(args.tmap));
  args.fixed_blocks = ((fixed_ok || (tmap && tmap_fixed)) && nw == nwc) ? 1u : 0u;
  args.bars_off = args.red_off + red_bytes;
  args.ncol = ncol;
  args.fb = fb;
  args.ksplit = 1;
  args.row_unit = d.epilogue != KQ_EPILOGUE_NONE ? 2 : 1;
  args.prologue = d.prologue;
  args.epilogue = d.epilogue;
  args.flags = d.flags;
  args.eps = d.eps;
  args.pair_scale = d.pair_scale;
  const uint32_t smem = args.bars_off + 2 * 8 * 8 + 128;

  plan.args = args;
  plan.mode = mode;
  plan.smem = smem;
  plan.grid = static_cast<uint32_t>(std::min<uint64_t>(ctx->sm_count, units));
  plan.block = (nw + 1) * 32;
  return KQ_OK;
}

cudaError_t launch(const void* fn, uint32_t grid, uint32_t block, uint32_t smem, bool pdl,
                   cudaStream_t stream, void* arg) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* params[] = {arg};
  return cudaLaunchKernelExC(&cfg, fn, params);
}

std::string shape(uint32_t grid, uint32_t block, uint32_t smem) {
  return "grid " + std::to_string(grid) + " x " + std::to_string(block) + " threads, " +
         std::to_string(smem) + " B shared";
}

// Does the layout of b match a's (ring, tiles, shared-memory regions, warps)?
bool same_layout(const WarpMmaArgs& a, const WarpMmaArgs& b) {
  return a.row_bytes == b.row_bytes && a.nb == b.nb && a.nkt == b.nkt && a.nw == b.nw &&
         a.ring == b.ring && a.slot_bytes == b.slot_bytes && a.seg_bytes == b.seg_bytes &&
         a.table_off == b.table_off && a.mtable_off == b.mtable_off && a.ublk_off == b.ublk_off &&
         a.zero_off == b.zero_off && a.red_off == b.red_off && a.bars_off == b.bars_off &&
         a.row_perm == b.row_perm && a.split_tile == b.split_tile &&
         a.fixed_blocks == b.fixed_blocks && a.ncol == b.ncol && a.fb == b.fb &&
         a.ksplit == b.ksplit && a.tmap_mode == b.tmap_mode && a.tile_pitch == b.tile_pitch &&
         a.xpart == b.xpart;
}

}  // namespace

int warpmma_matvec(kq_ctx* ctx, const kq_matvec_desc& d, uint64_t ldx, uint64_t ldy,
                   cudaStream_t stream) {
  WarpMmaPlan plan;
  int rc = warpmma_plan(ctx, d, ldx, ldy, "kq_matvec", plan);
  if (rc) return rc;
  const cudaError_t e = launch(kVariants[plan.args.xpart ? kXPartVariant : plan.mode].fn, plan.grid, plan.block, plan.smem,
                               !(d.flags & KQ_FLAG_NO_PDL), stream, &plan.args);
  if (e != cudaSuccess)
    return cuda_fail(e, "cudaLaunchKernelExC", "warp-MMA matvec " + shape(plan.grid, plan.block, plan.smem));
  return KQ_OK;
}

int warpmma_plan_launch(kq_ctx* ctx, const kq_matvec_desc& d, kq_launch& out) {
  const char* call = "kq_matvec_plan";
  int rc = check_desc(d, call);
  if (rc) return rc;
  if (!warpmma_supports(d) || (d.flags & (KQ_FLAG_TENSOR_CORES | KQ_FLAG_CUDA_CORES)))
    return fail(KQ_E_UNSUPPORTED, call, "the warp-MMA kernel serves Q4_K batch 1..8 and Q5_K, Q6_K batch 1");
  const bool pair = d.epilogue != KQ_EPILOGUE_NONE;
  const uint64_t ldx = d.ldx ? d.ldx : d.k;
  const uint64_t ldy = d.ldy ? d.ldy : (pair ? d.rows / 2 : d.rows);
  WarpMmaPlan plan;
  rc = warpmma_plan(ctx, d, ldx, ldy, call, plan);
  if (rc) return rc;
  // the function's name, as the driver has it (the image is the same source, compiled alike)
  cudaFunction_t f = nullptr;
  cudaError_t e = cudaGetFuncBySymbol(&f, kVariants[plan.args.xpart ? kXPartVariant : plan.mode].fn);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetFuncBySymbol", call);
  using GetName = CUresult (*)(const char**, CUfunction);
  void* fp = nullptr;
  cudaDriverEntryPointQueryResult q;
  e = cudaGetDriverEntryPoint("cuFuncGetName", &fp, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fp)
    return fail(KQ_E_UNSUPPORTED, call, "the driver has no cuFuncGetName");
  const char* name = nullptr;
  const CUresult r = reinterpret_cast<GetName>(fp)(&name, reinterpret_cast<CUfunction>(f));
  if (r != CUDA_SUCCESS || !name || std::strlen(name) >= sizeof(out.kernel))
    return fail(KQ_E_UNSUPPORTED, call, "cuFuncGetName gave no usable name");
  static_assert(sizeof(WarpMmaArgs) <= sizeof(out.params), "kq_launch params too small");
  std::memset(&out, 0, sizeof(out));
  std::strcpy(out.kernel, name);
  out.grid[0] = plan.grid;
  out.grid[1] = out.grid[2] = 1;
  out.block[0] = plan.block;
  out.block[1] = out.block[2] = 1;
  out.shared_bytes = plan.smem;
  out.param_bytes = sizeof(WarpMmaArgs);
  std::memcpy(out.params, &plan.args, sizeof(WarpMmaArgs));
  return KQ_OK;
}

int tagged_unpack(kq_ctx* ctx, uint64_t dst, uint64_t src, uint64_t n, uint64_t epoch, uint64_t mul,
                  uint64_t add, cudaStream_t stream) {
  const char* call = "kq_tagged_unpack";
  if (!dst || !src || !epoch || dst % 4 || src % 8 || epoch % 8)
    return fail(KQ_E_INVALID, call, "dst 4-byte, src and epoch 8-byte aligned, non-null");
  if (n == 0) return KQ_OK;
  const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>((n + 255) / 256, uint64_t(ctx->sm_count) * 2));
  tagged_unpack_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<float*>(dst),
                                                 reinterpret_cast<const unsigned long long*>(src), n,
                                                 reinterpret_cast<const unsigned long long*>(epoch),
                                                 mul, add, ctx->err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernel", call);
  return KQ_OK;
}

int warpmma_push(kq_ctx* ctx, const kq_matvec_desc& d, const kq_push_desc& push, uint64_t ldx,
                 uint64_t ldy, cudaStream_t stream) {
  const char* call = "kq_matvec_push";
  WarpMmaPlan plan;
  // (the plan sizes its slots for the rows a CTA gets, which split K multiplies)
  // (the fixed-block loop on tensor-map tiles: Q6_K only, and not with split-K slots; the Q4_K
  // and Q5_K push kernels are compiled without it, which cost them registers)
  const uint32_t ks = std::min<uint32_t>(std::max<uint32_t>(push.ksplit, 1), 8);
  const bool tagged = (push.flags & KQ_PUSH_TAGGED) != 0;
  const bool tx = tagged && (push.wait_counter || (push.flags & KQ_PUSH_TAGGED_X));
  // (x in two parts only for a plain x: with a tagged x, the second part's table waits for its
  // loads with no tiles to hide them, and measured slower on B200 than the whole table)
  int rc = warpmma_plan(ctx, d, ldx, ldy, call, plan, ks, true,
                        d.type == KQ_TYPE_Q6_K && push.x_slots <= 1, !tx);
  if (rc) return rc;
  if (plan.mode != (d.type == KQ_TYPE_Q4_K ? 4 : d.type == KQ_TYPE_Q5_K ? 6 : 5))
    return fail(KQ_E_UNSUPPORTED, call, "k " + std::to_string(d.k) + " does not fit the integer kernel");
  PushArgs q = {};
  q.y.wait_cnt = reinterpret_cast<const unsigned long long*>(push.wait_counter);
  q.y.npush = push.npush;
  q.y.push_rows = push.npush ? push.push_rows : 0;
  for (uint32_t r = 0; r < kChainMaxRanks; ++r) {
    q.y.push_y[r] = r < push.npush ? reinterpret_cast<float*>(push.y[r]) : nullptr;
    q.y.counter[r] = r < push.npush ? reinterpret_cast<unsigned long long*>(push.counter[r]) : nullptr;
  }
  q.epoch = reinterpret_cast<const unsigned long long*>(push.epoch);
  q.wait_mul = push.wait_mul;
  q.wait_add = push.wait_add;
  q.y.tagged = tagged ? 1u : 0u;
  q.push_mul = push.push_mul;
  q.push_add = push.push_add;
  q.x_slots = push.x_slots ? push.x_slots : 1u;
  const uint32_t ksplit = push.ksplit ? push.ksplit : 1u;
  if (ksplit > 1 || q.x_slots > 1) {
    if (!tagged) return fail(KQ_E_INVALID, call, "split K and x slots go with tagged pushes");
    if (q.x_slots > 8 || ksplit > 8 || (ksplit & (ksplit - 1)))
      return fail(KQ_E_INVALID, call, "ksplit must be 1, 2, 4 or 8 and x_slots 1..8");
    if (q.x_slots > 1 && !tx) return fail(KQ_E_INVALID, call, "x slots need a tagged x");
    if (ksplit > plan.args.nkt)
      return fail(KQ_E_INVALID, call, "ksplit " + std::to_string(ksplit) + " above the " +
                                          std::to_string(plan.args.nkt) + " K-tiles of a row");
    if (ksplit > 1 && d.epilogue != KQ_EPILOGUE_NONE)
      return fail(KQ_E_INVALID, call, "split K sums its parts in the reader: no product epilogue");
  }
  plan.args.ksplit = ksplit;
  q.y.out_slot = push.npush * push.push_rows;  // a slot is a whole full vector
  if (ksplit > 1) {
    // every row range is shared by ksplit CTAs: whole groups of them
    const uint64_t units = d.epilogue != KQ_EPILOGUE_NONE ? d.rows / 2 : d.rows;
    plan.grid = static_cast<uint32_t>(std::min<uint64_t>(ctx->sm_count / ksplit, units)) * ksplit;
  }
  if (tagged) {
    q.y.wait_cnt = nullptr;
    for (uint32_t r = 0; r < kChainMaxRanks; ++r) q.y.counter[r] = nullptr;
    if (!push.epoch || push.epoch % 8)
      return fail(KQ_E_INVALID, call, "tagged pushes need an 8-byte aligned epoch");
    for (uint32_t r = 0; r < push.npush; ++r)
      if (push.y[r] % 8) return fail(KQ_E_INVALID, call, "tagged vectors must be 8-byte aligned");
    if (tx && (d.x % 16 || d.ldx > d.k))
      return fail(KQ_E_INVALID, call, "a tagged x must be 16-byte aligned, batch 1");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(plan.block);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (d.flags & KQ_FLAG_NO_PDL) ? 0 : 1;
  void* params[] = {&plan.args, &q};
  const cudaError_t e =
      cudaLaunchKernelExC(&cfg, push_fn(d.type, !tx ? 0 : q.x_slots > 1 ? 2 : 1, plan.args.xpart != 0), params);
  if (e != cudaSuccess)
    return cuda_fail(e, "cudaLaunchKernelExC", "warp-MMA push " + shape(plan.grid, plan.block, plan.smem));
  return KQ_OK;
}

int warpmma_chain(kq_ctx* ctx, const kq_chain_job* jobs, uint32_t njobs, uint64_t epoch,
                  cudaStream_t stream) {
  const char* call = "kq_matvec_chain";
  if (!jobs || njobs == 0 || njobs > kChainMaxJobs)
    return fail(KQ_E_INVALID, call, "1.." + std::to_string(kChainMaxJobs) + " jobs");
  if (!epoch || epoch % 8) return fail(KQ_E_INVALID, call, "epoch must be a non-null 8-byte aligned address");
  ChainParams p = {};
  p.epoch = reinterpret_cast<const unsigned long long*>(epoch);
  p.njobs = njobs;
  uint32_t smem = 0, block = 0;
  for (uint32_t j = 0; j < njobs; ++j) {
    const kq_chain_job& job = jobs[j];
    const kq_matvec_desc& d = job.mv;
    const std::string at = "job " + std::to_string(j) + ": ";
    int rc = check_desc(d, call);
    if (rc) return rc;
    if (d.type != jobs[0].mv.type || d.k != jobs[0].mv.k)
      return fail(KQ_E_INVALID, call, at + "every job of a chain has the first job's type and k");
    if (d.batch != 1 || (d.type != KQ_TYPE_Q4_K && d.type != KQ_TYPE_Q5_K && d.type != KQ_TYPE_Q6_K))
      return fail(KQ_E_INVALID, call, at + "chains take batch-1 Q4_K, Q5_K or Q6_K matvecs");
    if (d.ldx > d.k || d.ldy > (d.epilogue != KQ_EPILOGUE_NONE ? d.rows / 2 : d.rows))
      return fail(KQ_E_INVALID, call, at + "batch 1 has no strides");
    if (d.flags & (KQ_FLAG_TENSOR_CORES | KQ_FLAG_CUDA_CORES | kFlagAltBatch1 | kFlagWarpPerBlock))
      return fail(KQ_E_INVALID, call, at + "chains run the warp-MMA integer kernel only");
    if (job.npush > kChainMaxRanks) return fail(KQ_E_INVALID, call, at + "npush above 8");
    const uint32_t outs = d.epilogue != KQ_EPILOGUE_NONE ? d.rows / 2 : d.rows;
    if (job.npush && (job.push_rows == 0 || job.push_rows > outs))
      return fail(KQ_E_INVALID, call, at + "push_rows must be 1..the job's outputs");
    for (uint32_t r = 0; r < job.npush; ++r)
      if (!job.push_y[r] || job.push_y[r] % 4 || !job.counter[r] || job.counter[r] % 8)
        return fail(KQ_E_INVALID, call, at + "push_y must be 4-byte and counter 8-byte aligned, non-null");
    if (!job.npush && job.counter[0] % 8) return fail(KQ_E_INVALID, call, at + "counter must be 8-byte aligned");
    if (job.wait_counter % 8) return fail(KQ_E_INVALID, call, at + "wait_counter must be 8-byte aligned");
    WarpMmaPlan plan;
    rc = warpmma_plan(ctx, d, d.k, outs, call, plan, 1, false);
    if (rc) return rc;
    if (plan.mode != (d.type == KQ_TYPE_Q4_K ? 4 : d.type == KQ_TYPE_Q5_K ? 6 : 5))
      return fail(KQ_E_UNSUPPORTED, call, at + "k " + std::to_string(d.k) + " does not fit the integer kernel");
    if (j == 0)
      p.lay = plan.args;
    else if (!same_layout(p.lay, plan.args))
      return fail(KQ_E_UNSUPPORTED, call, at + "its tiles differ from the first job's");
    const WarpMmaArgs& g = plan.args;
    p.job[j] = JobArgs{g.W, g.x, g.y, g.total_bytes, g.rows, g.row_unit, g.prologue, g.epilogue,
                       g.eps, g.pair_scale};
    smem = plan.smem;
    block = plan.block;
    ChainSync& y = p.sync[j];
    y.wait_cnt = reinterpret_cast<const unsigned long long*>(job.wait_counter);
    y.wait_target = job.wait_target;
    y.npush = job.npush;
    y.push_rows = job.npush ? job.push_rows : 0;
    for (uint32_t r = 0; r < kChainMaxRanks; ++r) {
      y.push_y[r] = r < job.npush ? reinterpret_cast<float*>(job.push_y[r]) : nullptr;
      y.counter[r] = (r < job.npush || (r == 0 && !job.npush))
                         ? reinterpret_cast<unsigned long long*>(job.counter[r])
                         : nullptr;
    }
  }
  // one CTA per SM for every job: the CTAs wait on one another between jobs
  const uint32_t grid = static_cast<uint32_t>(ctx->sm_count);
  const cudaError_t e = launch(chain_fn(jobs[0].mv.type), grid, block, smem,
                               !(jobs[0].mv.flags & KQ_FLAG_NO_PDL), stream, &p);
  if (e != cudaSuccess)
    return cuda_fail(e, "cudaLaunchKernelExC", "warp-MMA chain " + shape(grid, block, smem));
  return KQ_OK;
}

}  // namespace kq
