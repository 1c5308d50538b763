// S1: the int4 W4A16 product fused with the per-row multi-LoRA update, tcgen05 + TMA (sm_100a), persistent.
//
// y (M, out) = bf16( x (M, K) . W^T + mid . B[a]^T ), W = bf16(fp32(u - z) * fp32(s)) from int4 words in the kernel
// layout (jb_int4_repack of the reference's layout: within each word the nibbles of inputs 0,2,4,6,1,3,5,7, so one
// shift and one mask give two neighbouring inputs), scales/zeros (K/G, columns) bf16.
//
// One CTA per SM loops over 256 x 128 output tiles (two 128-row halves sharing every dequantised weight tile), tile
// index n-tile major so concurrent CTAs share weight tiles in L2. 14 warps:
//   warp 0       TMA producer: per 64-wide K block the x tile (256 x 64 bf16, 128B swizzle), the packed words
//                (8 x 128 int32) and the group's scale (and zero) row into a STAGES-deep ring (mbarrier full[s]);
//   warp 1       allocates 512 TMEM columns (two 256-column accumulators, so a tile's epilogue overlaps the next
//                tile's main loop); one thread issues tcgen05.mma (M=128, N=128, K=16) x 4 x 2 per K block;
//   warps 2-9    two groups of four, each on alternate K blocks (two stages dequantised at once): each stage's
//                words into bf16 in the UMMA 128B-swizzled K-major layout (deq[s]).
// The LoRA expand runs as extra K blocks of the same accumulator. With one adapter per 128-row half (rows whose
// length is a multiple of 128 tokens) the producer loads each half's mid rows and its adapter's B rows by TMA as
// planes of 8 columns, and each half's expand is an MMA of its own. Otherwise (any other row length, down to one
// adapter id per token for packed requests of mixed lengths) the dequantisers gather the operands: the tile's
// distinct adapters, in pool-row order, each own `rank` expand columns; the x slot holds each row's mid in its
// adapter's block (zeros elsewhere: exact) and the weight slot those adapters' B rows. The tile's adapter set comes
// from a bitmask over pool rows per 256-row tile, built once at kernel start, so every role derives the
// same number of expand blocks for a tile. Every block starts at a multiple of 16 expand columns, so a row's own
// terms meet the tensor core in the same K16 positions whichever adapters share its tile: its bits do not depend
// on the other rows of the pass.
//   warps 10-13  epilogue: TMEM -> registers -> bf16 -> 16-byte stores of each row (clipped to M x out), then the
//                accumulator is released (tmem_empty). With `swiglu` the 128 columns are 64 gate | 64 up columns of
//                the interleaved gate/up group and the tile's 64 outputs are bf16(bf16(silu(g)) u) (the reference's
//                silu_mul, fast_path.py:141-156, on the rounded products).
// The base product is summed in fp32 in K order; the LoRA term joins the same fp32 accumulator; one rounding at the
// end: the reference's cut-product rule (int4_kernels.py:1-30). No atomics: the result is deterministic.
//
// Dequantisation: a nibble pair becomes bf16 (128 + u) by OR-ing the exponent bits 0x4300, minus (128 + z) is the
// exact small integer u - z, times the scale in one bf16 multiply (a single rounding of an exact product), which is
// bf16(fp32(u - z) * fp32(s)) bit for bit.

namespace jb {
namespace w4 {

// Stage trace (built only with -DJB_TRACE, `python -m jeff_b200.build --trace`): CTA 0 stamps clock64() at every
// hand-off of its first 256 K blocks into g_stage_trace[event][k block]: 0 producer saw the stage free, 1 its TMA
// loads issued, 2 / 3 the first warp of the K block's dequantiser group saw it full / arrived dequantised, 4 the
// MMA thread's waits returned, 5 its MMAs and commit issued, 6 / 7 the epilogue started / finished tile `it`, 8..11
// each dequantiser warp arrived, 12..15 each dequantiser warp saw the stage full. jb_stage_trace_read copies it out.
// Without JB_TRACE the stamps compile to nothing.
#ifdef JB_TRACE
__device__ unsigned long long g_prod_trace[6][256];
#define JB_PROD(ev, kg)                                                                    \
  do {                                                                                     \
    if (blockIdx.x == 0 && (unsigned)(kg) < 256u) g_prod_trace[ev][kg] = clock64();        \
  } while (0)
__device__ unsigned long long g_stage_trace[16][256];
#define JB_STAGE(ev, kg)                                                                   \
  do {                                                                                     \
    if (blockIdx.x == 0 && (unsigned)(kg) < 256u) g_stage_trace[ev][kg] = clock64();       \
  } while (0)
#else
#define JB_PROD(ev, kg) \
  do {                  \
  } while (0)
#define JB_STAGE(ev, kg) \
  do {                   \
  } while (0)
#endif

constexpr int BM = 256;             // rows per tile (two UMMA halves of 128)
constexpr int HM = 128;             // rows per half
constexpr int BN = 128;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int GROUPS = 2;          // dequantiser groups, each on alternate K blocks
constexpr int DEQ_WARPS = 8;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 64 + (DEQ_WARPS + EPI_WARPS) * 32;
constexpr int MASK_WORDS = 8;       // gathered expand: a tile's adapter set as a bitmask over pool rows < 256
constexpr int MAX_MASK_TILES = 128; // ... for up to 128 row tiles (m <= 32768)

struct Params {
  int M, K, columns, out, group;
  const __nv_bfloat16* mid;      // (M, rank) or null
  const __nv_bfloat16* lora_b;   // (pool_rows, columns, rank)
  const int* adapters;
  int rank, row_len, pool_rows;
  int swiglu;                    // 1: columns are interleaved gate|up blocks of 64; y holds silu(g) u, out/2 wide
  int m_tiles, n_tiles;
  __nv_bfloat16* y;
  int ldy;
  int* err;
  int planes3d;                  // 1: tm_mid / tm_lb load every plane of a half at once; 0: one plane per load
  int x_rows;                    // rows of tm_x's box: min(256, M rounded up to 16)
  // split K: each tile's K blocks in k_split equal slices, each slice a work item of its own. A slice writes its
  // fp32 sums to partials ([slice][column][token], ldp tokens per column), then bumps counters[tile]; the CTA whose
  // slice arrives last adds the slices in slice order (deterministic), rounds and stores y, and resets the counter
  int k_split;
  float* partials;
  int* counters;
  int ldp;
};

// the MMA's N for a tile's tokens from m0: its real tokens rounded up to 16, at most `cap` (small passes multiply
// only the rows they have)
__device__ __forceinline__ int tile_tokens(int M, int m0, int cap) { return min(cap, ((M - m0 + 15) >> 4) << 4); }

struct Layout {
  static constexpr int X_BYTES = BM * BK * 2;      // 32 KB: two 128-row swizzled tiles back to back
  static constexpr int W_BYTES = BN * BK * 2;      // 16 KB
  static constexpr int RAW_BYTES = 8 * BN * 4;     // 4 KB
  static constexpr int SC_BYTES = BN * 2;
  static constexpr int OFF_X = 0;
  static constexpr int OFF_W = OFF_X + STAGES * X_BYTES;
  static constexpr int OFF_RAW = OFF_W + STAGES * W_BYTES;
  static constexpr int OFF_SC = OFF_RAW + STAGES * RAW_BYTES;
  static constexpr int OFF_ZR = OFF_SC + STAGES * SC_BYTES;
  static constexpr int OFF_BAR = OFF_ZR + STAGES * SC_BYTES;
  static constexpr int NBAR = 3 * STAGES + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_ADP = OFF_MISC + 16;
  static constexpr int MAX_ROWS = 512;            // adapter indices staged in shared memory (M / row_len rows)
  static constexpr int OFF_MASK = OFF_ADP + MAX_ROWS * 4;
  static constexpr int OFF_STG = OFF_MASK + MAX_MASK_TILES * MASK_WORDS * 4;   // epilogue staging, 32 tokens
  static constexpr int STG_PITCH = BN + 8;                                         // bf16 elements per token row
  static constexpr int BYTES = OFF_STG + 32 * STG_PITCH * 2;
  static constexpr int ALLOC = BYTES + 1024;       // room to align the base to 1024 B
  static_assert(ALLOC <= 227 * 1024, "shared memory");
};

// words in the kernel layout: nibble slot (j >> 1) + 4 (j & 1) holds input j of the word's eight
__host__ __device__ constexpr int kernel_slot(int j) { return (j >> 1) + 4 * (j & 1); }

// 8 weights of one kernel-layout word: bf16((u - z) * s) in input order, s2 = {s, s}, zb2 = {128 + z, 128 + z}
__device__ __forceinline__ uint4 dequant8(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 zb2) {
  uint32_t r[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    uint32_t t = ((w >> (4 * p)) & 0x000F000Fu) | 0x43004300u;   // inputs 2p, 2p + 1
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t);
    v = __hmul2(__hsub2(v, zb2), s2);
    r[p] = *reinterpret_cast<uint32_t*>(&v);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

__device__ __forceinline__ __nv_bfloat162 zero_pair(const __nv_bfloat16* zr, int n) {
  float z = zr ? __bfloat162float(zr[n]) : 8.0f;
  return __floats2bfloat162_rn(128.0f + z, 128.0f + z);
}

// a row tile's adapter set (MASK_WORDS words, bit a for pool row a): its size, the number of members below a, and
// its j-th member in increasing order (j < the size)
__device__ __forceinline__ int mask_count(const uint32_t* mask) {
  int d = 0;
#pragma unroll
  for (int w = 0; w < MASK_WORDS; ++w) d += __popc(mask[w]);
  return d;
}
__device__ __forceinline__ int mask_rank(const uint32_t* mask, int a) {
  int r = __popc(mask[a >> 5] & ((1u << (a & 31)) - 1u));
  for (int w = 0; w < (a >> 5); ++w) r += __popc(mask[w]);
  return r;
}
__device__ __forceinline__ int mask_nth(const uint32_t* mask, int j) {
  for (int w = 0; w < MASK_WORDS; ++w) {
    uint32_t m = mask[w];
    const int c = __popc(m);
    if (j < c) {
      for (int i = 0; i < j; ++i) m &= m - 1u;   // drop the j lowest members
      return 32 * w + __ffs(m) - 1;
    }
    j -= c;
  }
  return 0;
}

// silu(g) rounded to bf16, by the fast exponential and division intrinsics (their error, a few fp32 units in the last
// place, moves the rounded value by one bf16 step only when it lies that close to a rounding boundary)
__device__ __forceinline__ float silu_rounded(float g) { return round_bf(__fdividef(g, 1.0f + __expf(-g))); }

template <bool ZERO>
__global__ void __launch_bounds__(THREADS, 1)
    w4a16_lora_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                      const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
                      const __grid_constant__ CUtensorMap tm_mid, const __grid_constant__ CUtensorMap tm_lb,
                      Params p) {
  pdl_begin();
  using L = Layout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* deq = bars + STAGES;
  uint64_t* empty = bars + 2 * STAGES;
  uint64_t* tmem_full = bars + 3 * STAGES;       // [2]
  uint64_t* tmem_empty = tmem_full + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  volatile int* epi_ok = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nkb = p.K / BK;
  const bool has_lora = p.mid != nullptr && p.rank > 0;
  // rows whose length is a multiple of 128 tokens (one adapter per 128-row half): the producer loads each half's
  // mid rows and its adapter's B rows by TMA, and each half's expand is its own MMA of depth rank (both halves in
  // one K block when 2 rank <= 64, else one block each); otherwise the dequantisers gather the operands (below)
  const bool lora_tma = has_lora && p.row_len % HM == 0;
  const bool gathered = has_lora && !lora_tma;
  const bool halves_together = 2 * p.rank <= BK;
  const int tiles = p.m_tiles * p.n_tiles;
  const int S = p.k_split;                 // K slices per tile (1: none)
  const int items = tiles * S;             // work items (tile, slice), the slice fastest
  const int kbs = nkb / S;                 // base K blocks of one item
  int* s_adp = reinterpret_cast<int*>(smem + L::OFF_ADP);
  uint32_t* s_mask = reinterpret_cast<uint32_t*>(smem + L::OFF_MASK);   // [m tile][MASK_WORDS]
  if (lora_tma) {
    const int rows = (p.M + p.row_len - 1) / p.row_len;
    for (int i = threadIdx.x; i < rows && i < L::MAX_ROWS; i += blockDim.x) {
      const int a = p.adapters[i];
      s_adp[i] = (a >= 0 && a < p.pool_rows) ? a : -1;
    }
  }
  if (gathered) {
    // each row tile's adapter set: bit a of the tile's mask for every valid adapter a of a token in the tile. A warp
    // takes 32 consecutive request rows; of a run of lanes with the same (tile, adapter) only the first one sets the
    // bit, so packed requests cost one shared atomic per run.
    for (int i = threadIdx.x; i < p.m_tiles * MASK_WORDS; i += blockDim.x) s_mask[i] = 0;
    __syncthreads();
    const int rows = (p.M + p.row_len - 1) / p.row_len;
    for (int r0 = warp * 32; r0 < rows; r0 += blockDim.x) {
      const int r = r0 + lane;
      int a = r < rows ? p.adapters[r] : -1;
      if (a >= p.pool_rows) a = -1;
      const int t0 = a >= 0 ? r * p.row_len : 0;                // the row's first token (< M) ...
      const int t1 = a >= 0 ? t0 + min(p.row_len, p.M - t0) - 1 : 0;   // ... and its last
      const int key = a >= 0 ? (t0 / BM) * 256 + a : -1;
      const int prev = __shfl_up_sync(0xffffffffu, key, 1);
      if (a >= 0) {
        const uint32_t bit = 1u << (a & 31);
        if (lane == 0 || prev != key) atomicOr(&s_mask[(t0 / BM) * MASK_WORDS + (a >> 5)], bit);
        for (int mt = t0 / BM + 1; mt <= t1 / BM; ++mt) atomicOr(&s_mask[mt * MASK_WORDS + (a >> 5)], bit);
      }
    }
  }
  // the K blocks of a tile of row tile mt: the base product's, then the expand's
  auto lora_blocks = [&](int mt) -> int {
    if (lora_tma) return halves_together ? 1 : 2;
    if (!gathered) return 0;
    return (mask_count(s_mask + mt * MASK_WORDS) * p.rank + BK - 1) / BK;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&deq[s], DEQ_WARPS / GROUPS);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], EPI_WARPS);
    }
    *abort_flag = 0;
    *epi_ok = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_s);
    if (ZERO) prefetch_tmap(&tm_z);
    if (lora_tma) {
      prefetch_tmap(&tm_mid);
      prefetch_tmap(&tm_lb);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer
    if (lane == 0) {
      const uint32_t bytes = p.x_rows * BK * 2 + L::RAW_BYTES + L::SC_BYTES * (ZERO ? 2 : 1);
      uint32_t kg = 0;
      for (int item = blockIdx.x; item < items && !*abort_flag; item += gridDim.x) {
        const int tile = item / S, ks = item % S;
        const int m0 = (tile % p.m_tiles) * BM, n0 = (tile / p.m_tiles) * BN;
        const int nkt = kbs + (ks == S - 1 ? lora_blocks(tile % p.m_tiles) : 0);
        for (int kb = 0; kb < nkt; ++kb, ++kg) {
          const int s = kg % STAGES;
          if (!mbar_wait(&empty[s], ((kg / STAGES) & 1) ^ 1, abort_flag, p.err, 1)) break;
          JB_STAGE(0, kg);
          if (kb < kbs) {
            const int kgl = ks * kbs + kb;   // the K block in the whole product
            mbar_arrive_expect_tx(&full[s], bytes);
            JB_PROD(0, kg);
            tma_load_2d(smem + L::OFF_X + s * L::X_BYTES, &tm_x, &full[s], kgl * BK, m0);
            JB_PROD(1, kg);
            tma_load_2d(smem + L::OFF_RAW + s * L::RAW_BYTES, &tm_w, &full[s], n0, kgl * (BK / 8));
            JB_PROD(2, kg);
            tma_load_2d(smem + L::OFF_SC + s * L::SC_BYTES, &tm_s, &full[s], n0, (kgl * BK) / p.group);
            JB_PROD(3, kg);
            if (ZERO) tma_load_2d(smem + L::OFF_ZR + s * L::SC_BYTES, &tm_z, &full[s], n0, (kgl * BK) / p.group);
            JB_PROD(4, kg);
            JB_STAGE(1, kg);
          } else if (lora_tma) {
            // a LoRA block by TMA: for each of its halves, the half's mid rows (rank / 8 planes of 128 rows x 16 B)
            // into the x slot and its adapter's B rows for this column tile into the weight slot. Rows past m and
            // an invalid adapter read outside the tensors: zeros.
            const int h_lo = halves_together ? 0 : kb - kbs, h_hi = halves_together ? 2 : h_lo + 1;
            const int planes = p.rank / 8;
            mbar_arrive_expect_tx(&full[s], 2 * (h_hi - h_lo) * planes * 2048);
            for (int h = h_lo; h < h_hi; ++h) {
              uint8_t* xd = smem + L::OFF_X + s * L::X_BYTES + (h - h_lo) * (HM * 128);
              uint8_t* wd = smem + L::OFF_W + s * L::W_BYTES + (h - h_lo) * planes * 2048;
              const int row0 = m0 + h * HM;
              const int a = row0 < p.M ? s_adp[row0 / p.row_len] : -1;
              const int brow0 = a >= 0 ? a * p.columns + n0 : p.pool_rows * p.columns;
              if (p.planes3d) {
                tma_load_3d(xd, &tm_mid, &full[s], 0, row0, 0);
                tma_load_3d(wd, &tm_lb, &full[s], 0, brow0, 0);
              } else {
                for (int c = 0; c < planes; ++c) {
                  tma_load_2d(xd + c * 2048, &tm_mid, &full[s], 8 * c, row0);
                  tma_load_2d(wd + c * 2048, &tm_lb, &full[s], 8 * c, brow0);
                }
              }
            }
          } else {
            mbar_arrive(&full[s]);   // a LoRA block: the stage is free; the dequantisers fill it
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the whole warp runs the loop and computes the (warp-uniform) descriptors; one
    // elected lane issues the MMAs and commits
    {
      // swap AB: the dequantised weights are A (M = 128 columns), the tokens B (N = 256 rows), so one MMA per K16
      // step covers the whole 256 x 128 tile and reads the weight tile once
      const bool issuer = elect_one();
      uint32_t kg = 0;
      int it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x, ++it) {
        const int tile = item / S, ks = item % S;
        const int b = it & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&tmem_empty[b], ((it >> 1) & 1) ^ 1, abort_flag, p.err, 2));
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * BM;
        const int m0 = (tile % p.m_tiles) * BM;
        const uint32_t idesc_tile = idesc_bf16(BN, tile_tokens(p.M, m0, BM));
        const int nkt = kbs + (ks == S - 1 ? lora_blocks(tile % p.m_tiles) : 0);
        for (int kb = 0; kb < nkt; ++kb, ++kg) {
          const int s = kg % STAGES;
          const uint32_t ph = (kg / STAGES) & 1;
          // one wait: the dequantisers arrive on deq[s] only after each of them saw full[s] complete (the stage's
          // TMA bytes landed), so deq[s] covers both
          ok = __all_sync(0xffffffffu, mbar_wait(&deq[s], ph, abort_flag, p.err, 4));
          if (!ok) break;
          if (issuer) JB_STAGE(4, kg);
          tc_fence_after();
          if (kb >= kbs && lora_tma) {
            // each half against its own adapter, planes layout: K16 step j reads planes 2j, 2j + 1
            const int h_lo = halves_together ? 0 : kb - kbs, h_hi = halves_together ? 2 : h_lo + 1;
            for (int h = h_lo; h < h_hi; ++h) {
              if (m0 + h * HM >= p.M) continue;   // a half past the pass's tokens adds nothing
              const uint32_t idesc_h = idesc_bf16(BN, tile_tokens(p.M, m0 + h * HM, HM));
              const uint32_t xa = smem_u32(smem + L::OFF_X + s * L::X_BYTES + (h - h_lo) * (HM * 128));
              const uint32_t wa = smem_u32(smem + L::OFF_W + s * L::W_BYTES + (h - h_lo) * (p.rank / 8) * 2048);
              for (int j = 0; j < p.rank / 16; ++j) {   // the half's 128 tokens are accumulator columns [128 h, +128)
                const uint64_t ad = planes_desc(wa + 2 * j * 2048, 2048), bd = planes_desc(xa + 2 * j * 2048, 2048);
                if (issuer) tc_mma_bf16(acc + h * HM, ad, bd, idesc_h, 1);
              }
            }
          } else {
            const uint64_t ad = sw128_desc(smem_u32(smem + L::OFF_W + s * L::W_BYTES));
            const uint64_t bd = sw128_desc(smem_u32(smem + L::OFF_X + s * L::X_BYTES));
            if (issuer) {
#pragma unroll
              for (int kk = 0; kk < BK / 16; ++kk)
                tc_mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, idesc_tile, (kb | kk) != 0);
            }
          }
          if (issuer) {
            tc_commit(&empty[s]);
            JB_STAGE(5, kg);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (issuer) tc_commit(&tmem_full[b]);
        __syncwarp();
      }
    }
  } else if (warp < 2 + DEQ_WARPS) {
    // ---------------- dequantisers: two groups of 128 threads, group g on the K blocks with kg % 2 == g
    const int et = threadIdx.x - 64;
    const int grp = et >> 7;
    const int n = et & (BN - 1);            // this thread's weight column
    uint32_t kg = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
      const int tile = item / S, ks = item % S;
      const int mt = tile % p.m_tiles;
      const int m0 = mt * BM, n0 = (tile / p.m_tiles) * BN;
      const int nkt = kbs + (ks == S - 1 ? lora_blocks(mt) : 0);
      for (int kb = 0; kb < nkt; ++kb, ++kg) {
        if ((int)(kg % GROUPS) != grp) continue;
        const int s = kg % STAGES;
        ok = mbar_wait(&full[s], (kg / STAGES) & 1, abort_flag, p.err, 5);
        if ((et & 127) == 0) JB_STAGE(2, kg);
        if (lane == 0) JB_STAGE(12 + ((et >> 5) & 3), kg);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        uint8_t* wt = smem + L::OFF_W + s * L::W_BYTES;
        if (kb < kbs) {
          const int32_t* raw = reinterpret_cast<const int32_t*>(smem + L::OFF_RAW + s * L::RAW_BYTES);
          const __nv_bfloat16* sc = reinterpret_cast<const __nv_bfloat16*>(smem + L::OFF_SC + s * L::SC_BYTES);
          const __nv_bfloat16* zr =
              ZERO ? reinterpret_cast<const __nv_bfloat16*>(smem + L::OFF_ZR + s * L::SC_BYTES) : nullptr;
          const __nv_bfloat162 s2 = __bfloat162bfloat162(sc[n]);
          const __nv_bfloat162 zb2 = zero_pair(zr, n);
          uint32_t w[8];
#pragma unroll
          for (int r = 0; r < 8; ++r) w[r] = static_cast<uint32_t>(raw[r * BN + n]);
#pragma unroll
          for (int r = 0; r < 8; ++r)
            *reinterpret_cast<uint4*>(wt + sw128_offset(n, r)) = dequant8(w[r], s2, zb2);
        } else if (!lora_tma) {
          // LoRA block, gathered: expand columns [col0, col0 + 64) of the tile's adapters in pool-row order, rank
          // columns each. Weight column n holds each block's adapter's B row; row lrow of each half puts its mid
          // in its adapter's block. The loads of each phase (B, then each half's mid) are issued before its stores,
          // so their latencies overlap.
          const uint32_t* mask = s_mask + mt * MASK_WORDS;
          const int ke = mask_count(mask) * p.rank;    // expand columns of this tile
          const int col0 = (kb - kbs) * BK;
          const int lrow = n;
          const int gn = n0 + n;
          uint4 v[8];
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            const int col = col0 + 8 * c8;
            v[c8] = make_uint4(0, 0, 0, 0);
            if (col < ke && gn < p.columns) {
              const int a = mask_nth(mask, col / p.rank);
              v[c8] = *reinterpret_cast<const uint4*>(p.lora_b + ((size_t)a * p.columns + gn) * p.rank +
                                                      (col % p.rank));
            }
          }
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) *reinterpret_cast<uint4*>(wt + sw128_offset(n, c8)) = v[c8];
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            const int gm = m0 + h * HM + lrow;
            int a = gm < p.M ? p.adapters[gm / p.row_len] : -1;
            if (a >= p.pool_rows) a = -1;
            const int lo = a >= 0 ? mask_rank(mask, a) * p.rank : 0;   // the row's block: [lo, lo + rank)
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) {
              const int col = col0 + 8 * c8;
              v[c8] = make_uint4(0, 0, 0, 0);
              if (a >= 0 && col >= lo && col < lo + p.rank)
                v[c8] = *reinterpret_cast<const uint4*>(p.mid + (size_t)gm * p.rank + (col - lo));
            }
            uint8_t* xt = smem + L::OFF_X + s * L::X_BYTES + h * (HM * 128);
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) *reinterpret_cast<uint4*>(xt + sw128_offset(lrow, c8)) = v[c8];
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&deq[s]);
        if ((et & 127) == 0) JB_STAGE(3, kg);
        if (lane == 0) JB_STAGE(8 + ((et >> 5) & 3), kg);
      }
    }
  } else {
    // ---------------- epilogue: 128 threads; thread = output column n of the tile (its TMEM lane), the accumulator's
    // 256 columns the tile's tokens. 32 tokens at a time: TMEM -> bf16 -> a [token][column] staging tile in shared
    // memory -> whole 16-byte pieces of each token's row to y (row-contiguous stores)
    const int et = threadIdx.x - 64 - DEQ_WARPS * 32;
    const int n = 32 * (warp & 3) + lane;
    const uint32_t lane_bits = (uint32_t)(32 * (warp & 3)) << 16;
    __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem + L::OFF_STG);
    __nv_bfloat16* y = p.y;
    const int ow = p.swiglu ? p.out / 2 : p.out;      // output columns
    volatile int* last_slice = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 12);
    int it = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x, ++it) {
      const int tile = item / S, ks = item % S;
      const int m0 = (tile % p.m_tiles) * BM, n0 = (tile / p.m_tiles) * BN;
      const int b = it & 1;
      if (et == 0) *epi_ok = mbar_wait(&tmem_full[b], (it >> 1) & 1, abort_flag, p.err, 6) ? 1 : 0;
      named_barrier(2, EPI_WARPS * 32);
      if (!*epi_ok) break;
      if (et == 0) JB_STAGE(6, it);
      tc_fence_after();
      const uint32_t acc = tmem + b * BM + lane_bits;
      const int t_end = min(BM, ((p.M - m0 + 31) >> 5) << 5);   // the tile's token chunks that hold tokens
      // 32 tokens t0 .. of column n (fp32 bits in r) -> bf16 staging -> y, by the staging tile
      auto emit = [&](int t0, const uint32_t (&r)[32]) {
#pragma unroll
        for (int e = 0; e < 32; ++e) stg[e * L::STG_PITCH + n] = f2bf(__uint_as_float(r[e]));
        named_barrier(2, EPI_WARPS * 32);
        if (!p.swiglu) {
#pragma unroll
          for (int i = et; i < 32 * (BN / 8); i += EPI_WARPS * 32) {
            const int tt = i / (BN / 8), c8 = i % (BN / 8);
            const int gm = m0 + t0 + tt, col = n0 + 8 * c8;
            if (gm < p.M && col < ow)
              *reinterpret_cast<uint4*>(y + (size_t)gm * p.ldy + col) =
                  *reinterpret_cast<const uint4*>(stg + tt * L::STG_PITCH + 8 * c8);
          }
        } else {
          // columns 0-63 of the tile are gate, 64-127 the matching up columns: 64 outputs bf16(bf16(silu(g)) u)
#pragma unroll
          for (int i = et; i < 32 * (BN / 16); i += EPI_WARPS * 32) {
            const int tt = i / (BN / 16), c8 = i % (BN / 16);
            const int gm = m0 + t0 + tt, col = n0 / 2 + 8 * c8;
            if (gm < p.M && col < ow) {
              const uint4 gv = *reinterpret_cast<const uint4*>(stg + tt * L::STG_PITCH + 8 * c8);
              const uint4 uv = *reinterpret_cast<const uint4*>(stg + tt * L::STG_PITCH + BN / 2 + 8 * c8);
              const uint32_t* gw = &gv.x;
              const uint32_t* uw = &uv.x;
              uint32_t ov[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                ov[e] = pack_bf2(silu_rounded(bf_lo(gw[e])) * bf_lo(uw[e]), silu_rounded(bf_hi(gw[e])) * bf_hi(uw[e]));
              *reinterpret_cast<uint4*>(y + (size_t)gm * p.ldy + col) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
            }
          }
        }
        named_barrier(2, EPI_WARPS * 32);
      };
      // this slice's partial sums of column n (split K only): [slice][column][token]
      float* part = S > 1 ? p.partials + ((size_t)ks * p.n_tiles * BN + n0 + n) * p.ldp + m0 : nullptr;
#pragma unroll 1
      for (int t0 = 0; t0 < t_end; t0 += 32) {
        uint32_t r[32];
        tmem_ld32(acc + t0, r);
        tc_wait_ld();
        if (t0 + 32 == t_end) {
          // the accumulator is read: release it to the MMA issuer for the tile after next
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tmem_empty[b]);
        }
        if (S == 1) {
          emit(t0, r);
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(part + t0 + 4 * q) =
                make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                            __uint_as_float(r[4 * q + 3]));
        }
      }
      if (S > 1) {
        // the last slice of the tile to arrive adds the slices in order and stores y
        __threadfence();
        named_barrier(2, EPI_WARPS * 32);
        if (et == 0) *last_slice = atomicAdd(&p.counters[tile], 1) == S - 1 ? 1 : 0;
        named_barrier(2, EPI_WARPS * 32);
        if (*last_slice) {
          __threadfence();
          const float* col_parts = p.partials + (size_t)(n0 + n) * p.ldp + m0;
          const size_t slice_stride = (size_t)p.n_tiles * BN * p.ldp;
#pragma unroll 1
          for (int t0 = 0; t0 < t_end; t0 += 32) {
            float sum[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(col_parts + t0 + 4 * q));
              sum[4 * q] = v.x; sum[4 * q + 1] = v.y; sum[4 * q + 2] = v.z; sum[4 * q + 3] = v.w;
            }
#pragma unroll 1
            for (int k2 = 1; k2 < S; ++k2) {
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float4 v =
                    __ldcg(reinterpret_cast<const float4*>(col_parts + k2 * slice_stride + t0 + 4 * q));
                sum[4 * q] += v.x; sum[4 * q + 1] += v.y; sum[4 * q + 2] += v.z; sum[4 * q + 3] += v.w;
              }
            }
            uint32_t r[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(sum[e]);
            emit(t0, r);
          }
          if (et == 0) p.counters[tile] = 0;   // ready for the next launch
        }
      }
      if (et == 0) JB_STAGE(7, it);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ LoRA first factor (mma.sync, small)
//
// mid (M, R) = bf16(x A[a]^T): one CTA of 4 warps per 16 rows; warp w sums inputs [w K / 4, (w + 1) K / 4) with
// bf16 mma.sync in fp32, four k-steps in flight; the four partial sums are added in warp order through shared
// memory (a fixed order: deterministic), rounded once.

template <int NB>   // rank / 8 output blocks
__global__ void __launch_bounds__(128) lora_shrink_kernel(const __nv_bfloat16* __restrict__ x, int M, int K,
                                                          const __nv_bfloat16* __restrict__ A, int pool_rows,
                                                          const int* __restrict__ adapters, int row_len,
                                                          __nv_bfloat16* __restrict__ mid) {
  pdl_begin();
  constexpr int R = NB * 8;
  __shared__ float part[4][16][R + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * 16;
  int a = adapters[m0 / row_len];
  if (a < 0 || a >= pool_rows) a = 0;
  const __nv_bfloat16* Aa = A + (size_t)a * R * K;
  const int g = lane >> 2, t = lane & 3;
  float acc[NB][4];
#pragma unroll
  for (int i = 0; i < NB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const __nv_bfloat16* x0 = x + (size_t)(m0 + g) * K;
  const __nv_bfloat16* x1 = x0 + (size_t)8 * K;
  const int kspan = K / 4;
  const int kbeg = warp * kspan, kend = kbeg + kspan;
#pragma unroll 4
  for (int k0 = kbeg; k0 < kend; k0 += 16) {
    const uint32_t a0 = *reinterpret_cast<const uint32_t*>(x0 + k0 + 2 * t);
    const uint32_t a1 = *reinterpret_cast<const uint32_t*>(x1 + k0 + 2 * t);
    const uint32_t a2 = *reinterpret_cast<const uint32_t*>(x0 + k0 + 8 + 2 * t);
    const uint32_t a3 = *reinterpret_cast<const uint32_t*>(x1 + k0 + 8 + 2 * t);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const __nv_bfloat16* brow = Aa + (size_t)(nb * 8 + g) * K + k0;
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(brow + 2 * t);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(brow + 8 + 2 * t);
      asm volatile(
          "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
          "{%0, %1, %2, %3};"
          : "+f"(acc[nb][0]), "+f"(acc[nb][1]), "+f"(acc[nb][2]), "+f"(acc[nb][3])
          : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
  }
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    const int col = nb * 8 + 2 * t;
    part[warp][g][col] = acc[nb][0];
    part[warp][g][col + 1] = acc[nb][1];
    part[warp][g + 8][col] = acc[nb][2];
    part[warp][g + 8][col + 1] = acc[nb][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * R; i += 128) {
    const int r = i / R, c = i % R;
    const float v = ((part[0][r][c] + part[1][r][c]) + part[2][r][c]) + part[3][r][c];
    mid[(size_t)(m0 + r) * R + c] = __float2bfloat16_rn(v);
  }
}

// ------------------------------------------------------------------ LoRA shrink, staged
//
// The same product in blocks of 32 rows (K a multiple of 128, any row length): 4 warps, warp w on rows 16 (w & 1)
// .. + 16 and on the K half w >> 1 of every 128-wide K step; the block's x rows and its adapter's A rows for each K
// step are staged in shared memory by cp.async (a four-deep ring) and read by ldmatrix. The two K halves' float32
// partials are added in a fixed order: deterministic. A block whose rows belong to several adapters (short rows,
// or one adapter id per token for packed requests of mixed lengths) runs the K loop once per distinct adapter and
// keeps each row from its own adapter's pass; every row goes through the same instructions in the same order
// either way, so its bits are those of a block of one adapter. Small blocks keep several CTAs resident per SM, so
// the loads of many blocks overlap.
constexpr int SH_ROWS = 32, SH_BK = 128, SH_PITCH = SH_BK + 8;   // 272-B rows: ldmatrix without bank conflicts
constexpr int SH_THREADS = 128;   // 4 warps: 2 groups of 16 rows x 2 halves of each 128-wide K step
constexpr int SH_STAGES = 4;      // cp.async ring: three K steps in flight while one is multiplied

__device__ __forceinline__ void sh_cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void sh_ldsm4(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void sh_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int NB>
constexpr int shrink_staged_smem() {
  return SH_STAGES * (SH_ROWS + NB * 8) * SH_PITCH * 2;
}

template <int NB>
__global__ void __launch_bounds__(SH_THREADS) lora_shrink_staged_kernel(const __nv_bfloat16* __restrict__ x, int M, int K,
                                                                 const __nv_bfloat16* __restrict__ A, int pool_rows,
                                                                 const int* __restrict__ adapters, int row_len,
                                                                 __nv_bfloat16* __restrict__ mid) {
  pdl_begin();
  constexpr int R = NB * 8;
  extern __shared__ __align__(16) uint8_t sh_smem[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(sh_smem);   // [SH_STAGES][SH_ROWS][SH_PITCH]
  __nv_bfloat16* as = xs + SH_STAGES * SH_ROWS * SH_PITCH;         // [SH_STAGES][R][SH_PITCH]
  float* red = reinterpret_cast<float*>(sh_smem);                  // after the K loop: [SH_ROWS][R + 4]
  __shared__ int row_adp[SH_ROWS], set[SH_ROWS], set_size;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rg = warp & 1, kh = warp >> 1;
  const int m0 = blockIdx.x * SH_ROWS;
  const int nk = K / SH_BK;
  // each row's adapter (an invalid one reads pool row 0; rows past M take row M - 1's) and the block's distinct
  // adapters in order of first appearance: one pass of the K loop per distinct adapter, each row kept from the
  // pass of its own, so a row's bits never depend on the rows that share its block
  if (warp == 0) {
    int a = adapters[min(m0 + lane, M - 1) / row_len];
    if (a < 0 || a >= pool_rows) a = 0;
    row_adp[lane] = a;
    const uint32_t peers = __match_any_sync(0xffffffffu, a);
    const bool first = (__ffs(peers) - 1) == lane;
    const uint32_t firsts = __ballot_sync(0xffffffffu, first);
    if (first) set[__popc(firsts & ((1u << lane) - 1u))] = a;
    if (lane == 0) set_size = __popc(firsts);
  }
  __syncthreads();
  for (int d = 0; d < set_size; ++d) {
    const int a = set[d];
    const __nv_bfloat16* Aa = A + (size_t)a * R * K;

    auto stage = [&](int kb, int buf) {
      const int k0 = kb * SH_BK;
      __nv_bfloat16* xd = xs + buf * SH_ROWS * SH_PITCH;
      __nv_bfloat16* ad = as + buf * R * SH_PITCH;
      for (int i = threadIdx.x; i < SH_ROWS * 16; i += SH_THREADS) {
        const int r = i >> 4, c = i & 15;
        const bool valid = m0 + r < M;
        sh_cp16(xd + r * SH_PITCH + c * 8, x + (size_t)(valid ? m0 + r : 0) * K + k0 + c * 8, valid);
      }
      for (int i = threadIdx.x; i < R * 16; i += SH_THREADS) {
        const int r = i >> 4, c = i & 15;
        sh_cp16(ad + r * SH_PITCH + c * 8, Aa + (size_t)r * K + k0 + c * 8, true);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };

    float acc[NB][4];
#pragma unroll
    for (int i = 0; i < NB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    // prologue: K steps 0 .. SH_STAGES - 2 in flight (an empty group where K runs out keeps the group count)
    for (int st = 0; st < SH_STAGES - 1; ++st) {
      if (st < nk) stage(st, st);
      else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int kb = 0; kb < nk; ++kb) {
      asm volatile("cp.async.wait_group %0;" ::"n"(SH_STAGES - 2) : "memory");   // step kb has landed
      __syncthreads();   // ... for every thread; and every warp is done with step kb - 1, whose buffer refills now
      if (kb + SH_STAGES - 1 < nk) stage(kb + SH_STAGES - 1, (kb + SH_STAGES - 1) % SH_STAGES);
      else asm volatile("cp.async.commit_group;" ::: "memory");
      const __nv_bfloat16* xb = xs + (kb % SH_STAGES) * SH_ROWS * SH_PITCH;
      const __nv_bfloat16* ab = as + (kb % SH_STAGES) * R * SH_PITCH;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int kc = kh * 64 + kk * 16;
        uint32_t af[4];
        sh_ldsm4(xb + (rg * 16 + (lane & 15)) * SH_PITCH + kc + (lane >> 4) * 8, af);
#pragma unroll
        for (int nb = 0; nb < NB; nb += 2) {
          const int i = lane >> 3;
          uint32_t bfr[4];
          sh_ldsm4(ab + (nb * 8 + (i >> 1) * 8 + (lane & 7)) * SH_PITCH + kc + (i & 1) * 8, bfr);
          sh_mma(acc[nb], af, bfr[0], bfr[1]);
          sh_mma(acc[nb + 1], af, bfr[2], bfr[3]);
        }
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();   // every warp is done with the staging buffers before the partials reuse them
    const int g = lane >> 2, t = lane & 3;
    constexpr int RP = R + 4;
    if (kh == 1) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const int col = nb * 8 + 2 * t;
        red[(rg * 16 + g) * RP + col] = acc[nb][0];
        red[(rg * 16 + g) * RP + col + 1] = acc[nb][1];
        red[(rg * 16 + g + 8) * RP + col] = acc[nb][2];
        red[(rg * 16 + g + 8) * RP + col + 1] = acc[nb][3];
      }
    }
    __syncthreads();
    if (kh == 0) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const int col = nb * 8 + 2 * t;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int row = rg * 16 + g + 8 * hf;
          if (m0 + row < M && row_adp[row] == a) {
            const float v0 = acc[nb][2 * hf] + red[row * RP + col];
            const float v1 = acc[nb][2 * hf + 1] + red[row * RP + col + 1];
            *reinterpret_cast<uint32_t*>(mid + (size_t)(m0 + row) * R + col) = pack_bf2(v0, v1);
          }
        }
      }
    }
    __syncthreads();   // the partials are read before the next pass stages into the same shared memory
  }
}

template <int NB>
int launch_shrink_staged(const __nv_bfloat16* x, int m, int k, const __nv_bfloat16* a, int pool_rows,
                         const int* adapters, int row_len, __nv_bfloat16* mid, cudaStream_t st) {
  constexpr int bytes = shrink_staged_smem<NB>();
  static_assert(bytes <= 227 * 1024, "shared memory");
  // set on every call: the attribute belongs to the current device
  cudaError_t e = cudaFuncSetAttribute(lora_shrink_staged_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       bytes);
  if (e != cudaSuccess) return status_of(e, "lora_shrink_staged_kernel: shared memory attribute");
  launch_pdl(lora_shrink_staged_kernel<NB>, (m + SH_ROWS - 1) / SH_ROWS, SH_THREADS, bytes, st, x, m, k, a, pool_rows, adapters,
                                                                                 row_len, mid);
  return check_launch("lora_shrink_staged_kernel");
}

// ------------------------------------------------------------------ standalone dequantiser (verification)

__global__ void int4_dequant_kernel(const int32_t* __restrict__ words, const __nv_bfloat16* __restrict__ scales,
                                    const __nv_bfloat16* __restrict__ zeros, int K, int columns, int group,
                                    __nv_bfloat16* __restrict__ out) {
  pdl_begin();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int i = blockIdx.y;   // word row: inputs 8i .. 8i + 7
  if (c >= columns) return;
  const int gi = (8 * i) / group;
  const __nv_bfloat162 s2 = __bfloat162bfloat162(scales[(size_t)gi * columns + c]);
  const float z = zeros ? __bfloat162float(zeros[(size_t)gi * columns + c]) : 8.0f;
  const __nv_bfloat162 zb2 = __floats2bfloat162_rn(128.0f + z, 128.0f + z);
  const uint4 v = dequant8(static_cast<uint32_t>(words[(size_t)i * columns + c]), s2, zb2);
  *reinterpret_cast<uint4*>(out + (size_t)c * K + 8 * i) = v;
}

template <bool ZERO>
int launch(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tz,
           const CUtensorMap& tm, const CUtensorMap& tl, const Params& p, cudaStream_t stream) {
  auto kernel = w4a16_lora_kernel<ZERO>;
  // queried on every call (well under a microsecond each): the attribute and the SM count belong to the current
  // device, and no per-device cache is shared between host threads
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return status_of(e, "w4a16: cudaGetDevice");
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout::ALLOC);
  if (e != cudaSuccess) return status_of(e, "w4a16: cudaFuncSetAttribute");
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return status_of(e, "w4a16: SM count");
  const int items = p.m_tiles * p.n_tiles * p.k_split;
  const int grid = items < sms ? items : sms;
  launch_pdl(kernel, grid, THREADS, Layout::ALLOC, stream, tx, tw, ts, tz, tm, tl, p);
  return check_launch("w4a16_lora_kernel");
}

// reference word layout (input 8i + j in bits 4j) -> kernel layout (input j in slot kernel_slot(j)); in place ok
__global__ void int4_repack_kernel(const int32_t* __restrict__ in, int32_t* __restrict__ out, size_t n) {
  pdl_begin();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t w = static_cast<uint32_t>(in[i]);
  uint32_t r = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) r |= ((w >> (4 * j)) & 0xFu) << (4 * kernel_slot(j));
  out[i] = static_cast<int32_t>(r);
}

}  // namespace w4
}  // namespace jb

#include "w4a16_tmem.cu"
#include "w4a16_small.cu"

using namespace jb;

extern "C" int jb_int4_dequant(const int32_t* words, const uint16_t* scales, const uint16_t* zeros, int k,
                               int columns, int group, uint16_t* out, void* stream) {
  JB_REQUIRE(words && scales && out, "jb_int4_dequant: null pointer");
  JB_REQUIRE(k > 0 && k % 64 == 0 && columns > 0 && columns % 64 == 0,
             "jb_int4_dequant: k (%d) and columns (%d) must be positive multiples of 64", k, columns);
  JB_REQUIRE(group == 64 || group == 128, "jb_int4_dequant: group %d (64 or 128)", group);
  JB_REQUIRE(k % group == 0, "jb_int4_dequant: k %d is not a multiple of the group %d", k, group);
  dim3 grid((columns + 127) / 128, k / 8);
  launch_pdl(w4::int4_dequant_kernel, grid, 128, 0, (cudaStream_t)stream,
      words, reinterpret_cast<const __nv_bfloat16*>(scales), reinterpret_cast<const __nv_bfloat16*>(zeros), k,
      columns, group, reinterpret_cast<__nv_bfloat16*>(out));
  return check_launch("int4_dequant_kernel");
}

extern "C" int jb_lora_shrink(const uint16_t* x, int m, int k, const uint16_t* lora_a, int rank, int pool_rows,
                              const int32_t* adapters, int row_len, uint16_t* mid, void* stream) {
  JB_REQUIRE(x && lora_a && adapters && mid, "jb_lora_shrink: null pointer");
  JB_REQUIRE(m > 0, "jb_lora_shrink: m %d must be positive", m);
  JB_REQUIRE(k > 0 && k % 64 == 0, "jb_lora_shrink: k %d must be a positive multiple of 64", k);
  JB_REQUIRE(row_len > 0, "jb_lora_shrink: row_len %d must be positive", row_len);
  JB_REQUIRE(pool_rows > 0, "jb_lora_shrink: pool_rows %d", pool_rows);
  auto xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto ab = reinterpret_cast<const __nv_bfloat16*>(lora_a);
  auto mb = reinterpret_cast<__nv_bfloat16*>(mid);
  cudaStream_t st = (cudaStream_t)stream;
  // the tcgen05 shrink (lora_shrink_tc.cu) for the pools the fast path builds (at most 256 rows); the mma.sync
  // kernels below for larger pools
  if (pool_rows <= lsh::MAX_POOL_ROWS && rank % 16 == 0 && rank >= 16 && rank <= 64) {
    JB_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(lora_a) |
                 reinterpret_cast<uintptr_t>(mid)) & 15) == 0,
               "jb_lora_shrink: x, lora_a and mid must be 16-byte aligned");
    return lsh::launch(xb, m, k, ab, rank, pool_rows, adapters, row_len, mb, st);
  }
  if (k % w4::SH_BK == 0) {
    switch (rank) {
      case 16: return w4::launch_shrink_staged<2>(xb, m, k, ab, pool_rows, adapters, row_len, mb, st);
      case 32: return w4::launch_shrink_staged<4>(xb, m, k, ab, pool_rows, adapters, row_len, mb, st);
      case 48: return w4::launch_shrink_staged<6>(xb, m, k, ab, pool_rows, adapters, row_len, mb, st);
      case 64: return w4::launch_shrink_staged<8>(xb, m, k, ab, pool_rows, adapters, row_len, mb, st);
      default: set_error("jb_lora_shrink: rank %d (16, 32, 48 or 64)", rank); return JB_EINVAL;
    }
  }
  // k not a multiple of 128: blocks of 16 rows of one adapter
  JB_REQUIRE(m % 16 == 0 && row_len % 16 == 0,
             "jb_lora_shrink: with k %d (not a multiple of 128), m %d and row_len %d must be multiples of 16", k, m,
             row_len);
  dim3 grid(m / 16);
  switch (rank) {
    case 16: launch_pdl(w4::lora_shrink_kernel<2>, grid, 128, 0, st, xb, m, k, ab, pool_rows, adapters, row_len, mb); break;
    case 32: launch_pdl(w4::lora_shrink_kernel<4>, grid, 128, 0, st, xb, m, k, ab, pool_rows, adapters, row_len, mb); break;
    case 48: launch_pdl(w4::lora_shrink_kernel<6>, grid, 128, 0, st, xb, m, k, ab, pool_rows, adapters, row_len, mb); break;
    case 64: launch_pdl(w4::lora_shrink_kernel<8>, grid, 128, 0, st, xb, m, k, ab, pool_rows, adapters, row_len, mb); break;
    default: set_error("jb_lora_shrink: rank %d (16, 32, 48 or 64)", rank); return JB_EINVAL;
  }
  return check_launch("lora_shrink_kernel");
}

namespace jb {
namespace w4 {
// jb_w4a16_lora with split K: k_split slices per tile (1: none), partials and counters the caller's scratch
// k_split < 0: the small-pass kernel (w4a16_small.cu) with -k_split - 1 slices (0: its own choice)
static int w4a16_lora_impl(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                           const uint16_t* zeros, int group, int columns, int out, const uint16_t* mid,
                           const uint16_t* lora_b, int rank, int pool_rows, const int32_t* adapters, int row_len,
                           uint16_t* y, int ldy, int flags, int k_split, float* partials, int32_t* counters,
                           void* stream) {
  const bool swiglu = (flags & JB_PRODUCT_SWIGLU) != 0;
  const int yw = swiglu ? out / 2 : out;   // output columns
  JB_REQUIRE(x && words && scales && y, "jb_w4a16_lora: null pointer");
  JB_REQUIRE(m > 0 && k > 0 && k % 64 == 0, "jb_w4a16_lora: m %d, k %d (k a multiple of 64)", m, k);
  JB_REQUIRE(columns > 0 && columns % 64 == 0 && out > 0 && out <= columns,
             "jb_w4a16_lora: columns %d (multiple of 64), out %d <= columns", columns, out);
  JB_REQUIRE(!swiglu || (columns % w4::BN == 0 && out == columns),
             "jb_w4a16_lora: the SwiGLU epilogue needs interleaved gate|up blocks filling whole 128-column tiles "
             "(columns %d, out %d)", columns, out);
  JB_REQUIRE(group == 64 || group == 128, "jb_w4a16_lora: group %d (64 or 128)", group);
  JB_REQUIRE(out % 8 == 0, "jb_w4a16_lora: out %d must be a multiple of 8", out);
  JB_REQUIRE(ldy >= yw && ldy % 8 == 0, "jb_w4a16_lora: ldy %d must be >= %d and a multiple of 8", ldy, yw);
  JB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(words) & 15) == 0 && (reinterpret_cast<uintptr_t>(scales) & 15) == 0,
             "jb_w4a16_lora: x, y, words and scales must be 16-byte aligned");
  const bool lora = mid != nullptr && rank > 0;
  if (lora) {
    JB_REQUIRE(lora_b && adapters, "jb_w4a16_lora: LoRA needs lora_b and adapters");
    JB_REQUIRE(rank % 16 == 0 && rank <= 64, "jb_w4a16_lora: rank %d (16, 32, 48 or 64)", rank);
    JB_REQUIRE(row_len > 0, "jb_w4a16_lora: row_len %d must be positive", row_len);
    JB_REQUIRE(pool_rows > 0, "jb_w4a16_lora: pool_rows %d", pool_rows);
    if (row_len % w4::HM) {   // the gathered expand: one adapter set per 256-row tile, kept in shared memory
      JB_REQUIRE(pool_rows <= 32 * w4::MASK_WORDS,
                 "jb_w4a16_lora: %d pool rows; with rows of %d tokens (not a multiple of 128) at most %d", pool_rows,
                 row_len, 32 * w4::MASK_WORDS);
      JB_REQUIRE((m + w4::BM - 1) / w4::BM <= w4::MAX_MASK_TILES,
                 "jb_w4a16_lora: m %d; with rows of %d tokens (not a multiple of 128) at most %d tokens", m, row_len,
                 w4::MAX_MASK_TILES * w4::BM);
    } else {
      JB_REQUIRE((m + row_len - 1) / row_len <= w4::Layout::MAX_ROWS, "jb_w4a16_lora: more than %d rows",
                 w4::Layout::MAX_ROWS);
    }
  }
  if (k_split < 0) {
    if (lora)
      JB_REQUIRE((reinterpret_cast<uintptr_t>(mid) & 15) == 0 && (reinterpret_cast<uintptr_t>(lora_b) & 15) == 0,
                 "jb_w4a16_lora: mid and lora_b must be 16-byte aligned");
    if (zeros) JB_REQUIRE((reinterpret_cast<uintptr_t>(zeros) & 15) == 0, "jb_w4a16_lora: zeros alignment");
    return w4s::launch(x, m, k, words, scales, zeros, group, columns, out, lora ? mid : nullptr, lora_b, rank,
                       pool_rows, adapters, row_len, y, ldy, swiglu, -k_split - 1, (cudaStream_t)stream);
  }
  // JB_PRODUCT_TMEM_A: the tensor-memory form (w4a16_tmem.cu), for calls whose LoRA rows are whole 128-token halves
  // (or one row for the whole pass); the same bits. Measured on a B200 at the Gated DeltaNet in_proj shape it takes
  // 245 us against 162 us for the shared-memory form below, so it is not the default.
  if ((flags & JB_PRODUCT_TMEM_A) && (!lora || row_len % w4t::HT == 0 || m <= row_len))
    return w4t::launch(x, m, k, words, scales, zeros, group, columns, out, mid, lora_b, rank, pool_rows, adapters,
                       row_len, y, ldy, swiglu, (cudaStream_t)stream);
  CUtensorMap tx, tw, ts, tz, tm, tl;
  int st;
  constexpr int BN = w4::BN;
  // small passes load only the rows they have: the box is the pass's tokens rounded up to 16, at most a tile
  const int x_rows = m < w4::BM ? ((m + 15) / 16) * 16 : w4::BM;
  if ((st = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k, m, (uint64_t)k * 2, 64, x_rows,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&tw, words, CU_TENSOR_MAP_DATA_TYPE_INT32, columns, k / 8, (uint64_t)columns * 4, BN, 8,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
    return st;
  if ((st = make_tmap_2d(&ts, scales, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, columns, k / group, (uint64_t)columns * 2,
                         BN, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return st;
  if (zeros) {
    JB_REQUIRE((reinterpret_cast<uintptr_t>(zeros) & 15) == 0, "jb_w4a16_lora: zeros must be 16-byte aligned");
    if ((st = make_tmap_2d(&tz, zeros, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, columns, k / group, (uint64_t)columns * 2,
                           BN, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
  } else {
    tz = ts;
  }
  if (lora) {
    JB_REQUIRE((reinterpret_cast<uintptr_t>(mid) & 15) == 0 && (reinterpret_cast<uintptr_t>(lora_b) & 15) == 0,
               "jb_w4a16_lora: mid and lora_b must be 16-byte aligned");
  }
  int planes3d = 0;
  if (lora && row_len % w4::HM == 0) {
    // the planes maps; where the driver refuses them, 2D maps of one plane per load
    planes3d = make_tmap_planes(&tm, mid, m, rank, (uint64_t)rank * 2, w4::HM) == JB_OK &&
               make_tmap_planes(&tl, lora_b, (uint64_t)pool_rows * columns, rank, (uint64_t)rank * 2, w4::BN) == JB_OK;
    if (!planes3d) {
      if ((st = make_tmap_2d(&tm, mid, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, m, (uint64_t)rank * 2, 8, w4::HM,
                             CU_TENSOR_MAP_SWIZZLE_NONE)))
        return st;
      if ((st = make_tmap_2d(&tl, lora_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, (uint64_t)pool_rows * columns,
                             (uint64_t)rank * 2, 8, w4::BN, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return st;
    }
  } else {
    tm = tx;
    tl = tx;
  }
  w4::Params p{m, k, columns, out, group,
               lora ? reinterpret_cast<const __nv_bfloat16*>(mid) : nullptr,
               reinterpret_cast<const __nv_bfloat16*>(lora_b), adapters, lora ? rank : 0, row_len > 0 ? row_len : 128,
               pool_rows, swiglu ? 1 : 0, (m + w4::BM - 1) / w4::BM, (columns + BN - 1) / BN,
               reinterpret_cast<__nv_bfloat16*>(y), ldy, device_status_word(), planes3d, x_rows,
               k_split, partials, counters, ((m + 31) / 32) * 32};
  if (zeros) return w4::launch<true>(tx, tw, ts, tz, tm, tl, p, (cudaStream_t)stream);
  return w4::launch<false>(tx, tw, ts, tz, tm, tl, p, (cudaStream_t)stream);
}
}  // namespace w4
}  // namespace jb

extern "C" int jb_w4a16_lora(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                             const uint16_t* zeros, int group, int columns, int out, const uint16_t* mid,
                             const uint16_t* lora_b, int rank, int pool_rows, const int32_t* adapters, int row_len,
                             uint16_t* y, int ldy, int flags, void* stream) {
  return w4::w4a16_lora_impl(x, m, k, words, scales, zeros, group, columns, out, mid, lora_b, rank, pool_rows,
                             adapters, row_len, y, ldy, flags, 1, nullptr, nullptr, stream);
}

extern "C" int jb_w4a16_lora_small(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                                   const uint16_t* zeros, int group, int columns, int out, const uint16_t* mid,
                                   const uint16_t* lora_b, int rank, int pool_rows, const int32_t* adapters,
                                   int row_len, uint16_t* y, int ldy, int flags, int split, void* stream) {
  JB_REQUIRE(split >= 0 && split <= w4s::MAX_SPLIT, "jb_w4a16_lora_small: split %d (0 to %d)", split,
             w4s::MAX_SPLIT);
  return w4::w4a16_lora_impl(x, m, k, words, scales, zeros, group, columns, out, mid, lora_b, rank, pool_rows,
                             adapters, row_len, y, ldy, flags, -split - 1, nullptr, nullptr, stream);
}

#ifdef JB_TRACE
// Measurement builds only (python -m jeff_b200.build --trace, libjeffb200_trace.so): copies the shared-memory
// product kernel's stage trace, 16 x 256 clock64() stamps of CTA 0's hand-offs in its last launch, to `out`. Not
// part of the product library or its header.
extern "C" int jb_prod_trace_read(uint64_t* out) {
  return status_of(cudaMemcpyFromSymbol(out, w4::g_prod_trace, sizeof(w4::g_prod_trace)), "jb_prod_trace_read");
}
extern "C" int jb_small_trace_read(uint64_t* out) {
  return status_of(cudaMemcpyFromSymbol(out, w4s::g_small_trace, sizeof(w4s::g_small_trace)), "jb_small_trace_read");
}
extern "C" int jb_small_span_read(uint64_t* out) {
  return status_of(cudaMemcpyFromSymbol(out, w4s::g_small_span, sizeof(w4s::g_small_span)), "jb_small_span_read");
}
extern "C" int jb_stage_trace_read(uint64_t* out) {
  JB_REQUIRE(out, "jb_stage_trace_read: null pointer");
  return status_of(cudaMemcpyFromSymbol(out, w4::g_stage_trace, sizeof(w4::g_stage_trace)),
                   "jb_stage_trace_read: copy");
}
#endif

extern "C" int jb_int4_repack(const int32_t* words, int32_t* out, int k, int columns, void* stream) {
  JB_REQUIRE(words && out, "jb_int4_repack: null pointer");
  JB_REQUIRE(k > 0 && k % 8 == 0 && columns > 0, "jb_int4_repack: k %d, columns %d", k, columns);
  const size_t n = (size_t)(k / 8) * columns;
  launch_pdl(w4::int4_repack_kernel, (unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream, words, out, n);
  return check_launch("int4_repack_kernel");
}

extern "C" int jb_int4_lora_product(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                                    const uint16_t* zeros, int group, int columns, int out, const uint16_t* lora_a,
                                    const uint16_t* lora_b, int rank, int pool_rows, const int32_t* adapters,
                                    int row_len, uint16_t* mid, uint16_t* y, int ldy, int flags, void* stream) {
  if (rank > 0) {
    JB_REQUIRE(mid && lora_a, "jb_int4_lora_product: LoRA needs lora_a and the mid scratch");
    int st = jb_lora_shrink(x, m, k, lora_a, rank, pool_rows, adapters, row_len, mid, stream);
    if (st) return st;
  }
  return jb_w4a16_lora(x, m, k, words, scales, zeros, group, columns, out, rank > 0 ? mid : nullptr, lora_b, rank,
                       pool_rows, adapters, row_len, y, ldy, flags, stream);
}

// The product with the base product's K split over several CTAs for passes too small to fill the GPU (their
// tiles fewer than the SMs): each tile's K blocks in equal slices, at least two blocks each, as many slices as keep
// the work items within twice the SM count and the partials within the caller's scratch. Same result as
// jb_int4_lora_product up to the order of the fp32 sums (slices added in slice order: deterministic).
extern "C" int jb_int4_lora_product_split(const uint16_t* x, int m, int k, const int32_t* words,
                                          const uint16_t* scales, const uint16_t* zeros, int group, int columns,
                                          int out, const uint16_t* lora_a, const uint16_t* lora_b, int rank,
                                          int pool_rows, const int32_t* adapters, int row_len, uint16_t* mid,
                                          uint16_t* y, int ldy, int flags, float* partials, int64_t partial_floats,
                                          int32_t* counters, int counter_count, void* stream) {
  JB_REQUIRE(partials && counters, "jb_int4_lora_product_split: null scratch");
  JB_REQUIRE((reinterpret_cast<uintptr_t>(partials) & 15) == 0, "jb_int4_lora_product_split: partials alignment");
  JB_REQUIRE(k > 0 && k % 64 == 0 && m > 0 && columns > 0, "jb_int4_lora_product_split: m %d, k %d, columns %d", m,
             k, columns);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int kb = k / 64;
  if (rank > 0) {
    JB_REQUIRE(mid && lora_a && adapters, "jb_int4_lora_product_split: LoRA needs lora_a, adapters and mid");
    // the shrink stays whole (slicing its K measured slower at 32 and 128 tokens)
    int st = jb_lora_shrink(x, m, k, lora_a, rank, pool_rows, adapters, row_len, mid, stream);
    if (st) return st;
  }
  // passes of at most 64 tokens in at most two LoRA rows: the weight-streaming kernel, its K slices one cluster
  if (!(flags & JB_PRODUCT_TMEM_A) && w4s::plan(m, k, columns, rank, row_len, group) > 0)
    return w4::w4a16_lora_impl(x, m, k, words, scales, zeros, group, columns, out, rank > 0 ? mid : nullptr, lora_b,
                               rank, pool_rows, adapters, row_len, y, ldy, flags, -1, partials, counters, stream);
  const int tiles = ((m + w4::BM - 1) / w4::BM) * ((columns + w4::BN - 1) / w4::BN);
  const int64_t ldp = ((m + 31) / 32) * 32;
  const int64_t per_slice = (int64_t)((columns + w4::BN - 1) / w4::BN) * w4::BN * ldp;
  // measured on a B200: slicing pays for few, long-K tiles of the smallest passes (32 tokens: out_proj 8 tiles x 32
  // K blocks 32 -> 25 us, down_proj 8 x 56 49 -> 31 us, both at 4 slices; more slices cost more) and costs where the
  // tiles already spread over half the SMs (in_proj, 65 tiles: 22 -> 27 us) or at 128 tokens, so only passes of at
  // most 64 tokens and at most a quarter as many tiles as SMs are sliced, into at most 4
  int split = 1;
  if (!(flags & JB_PRODUCT_TMEM_A) && m <= 64 && 4 * tiles <= sms && tiles <= counter_count) {
    for (int s = kb / 2 < 4 ? kb / 2 : 4; s >= 2; --s)
      if (kb % s == 0 && tiles * s <= 2 * sms && s * per_slice <= partial_floats) {
        split = s;
        break;
      }
  }
  return w4::w4a16_lora_impl(x, m, k, words, scales, zeros, group, columns, out, rank > 0 ? mid : nullptr, lora_b,
                             rank, pool_rows, adapters, row_len, y, ldy, flags, split, partials, counters, stream);
}

// ------------------------------------------------------------------ the product without caller scratch
//
// jb_int4_lora_product needs an (m, rank) bf16 scratch for the LoRA shrink's output. This variant takes none and
// allocates nothing: the scratch is a fixed array in the library's own device memory, sized for the largest pass
// the hot path runs (16384 tokens at rank 64). It serves callers that must not allocate device memory themselves:
// a host that binds the C ABI directly and owns no device allocator, or one whose device memory is reserved up
// front by its own pool. The array's address on each device is looked up once, by the first call made with that
// device current; make that first call before any stream capture. There is one array per device, so calls on one
// device must not overlap (two streams, or two host threads, at once): they would share the scratch and race.
// Nothing in the array has to start at zero: the shrink writes every element the expand then reads, on the same
// stream, before the expand launches.

static __device__ __align__(256) uint16_t g_product_mid[JB_PRODUCT_STATIC_MID_MAX];

static uint16_t* product_mid_scratch() {
  static std::mutex mu;
  static uint16_t* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    status_of(e, "jb_int4_lora_product_static: cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    set_error("jb_int4_lora_product_static: device %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_product_mid);
    if (e != cudaSuccess) {
      status_of(e, "jb_int4_lora_product_static: scratch address");
      return nullptr;
    }
    addr[dev] = static_cast<uint16_t*>(p);
  }
  return addr[dev];
}

extern "C" int jb_int4_lora_product_static(const uint16_t* x, int m, int k, const int32_t* words,
                                           const uint16_t* scales, const uint16_t* zeros, int group, int columns,
                                           int out, const uint16_t* lora_a, const uint16_t* lora_b, int rank,
                                           int pool_rows, const int32_t* adapters, int row_len, uint16_t* y, int ldy,
                                           int flags, void* stream) {
  uint16_t* mid = nullptr;
  if (rank > 0) {
    JB_REQUIRE(m > 0 && (long long)m * rank <= JB_PRODUCT_STATIC_MID_MAX,
               "jb_int4_lora_product_static: m %d x rank %d exceeds the static scratch of %d elements", m, rank,
               JB_PRODUCT_STATIC_MID_MAX);
    JB_REQUIRE(lora_a, "jb_int4_lora_product_static: LoRA needs lora_a");
    mid = product_mid_scratch();
    if (!mid) return JB_ECUDA;
  }
  return jb_int4_lora_product(x, m, k, words, scales, zeros, group, columns, out, lora_a, lora_b, rank, pool_rows,
                              adapters, row_len, mid, y, ldy, flags, stream);
}
