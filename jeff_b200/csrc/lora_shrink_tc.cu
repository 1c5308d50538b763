// The LoRA first factor on tcgen05: mid (M, R) = bf16(x A[a]^T), a = adapters[t / row_len] of token t (an invalid
// adapter index reads pool row 0, the zero adapter), the reference's lora_add first product
// (engine/fast_path.py:277-289) for every token of a pass at once.
//
// One CTA per 128 tokens (the MMA's M = 128 TMEM lanes). The tile's distinct adapters, in pool-row order, run in
// passes of COLS / R adapters: per 64-wide K block the producer (warp 4, one lane) loads the x tile (128 x 64,
// 128-byte swizzle) and each adapter's A rows (R x 64) by TMA into a STAGES-deep ring; the MMA warp (warp 5, one
// elected lane) issues, for each adapter j of the pass, an M 128 x N R MMA per K16 step into TMEM columns
// [j R, j R + R); the four epilogue warps (thread = token) read the columns of their own token's adapter, round once
// to bf16 and store the token's R values. Every adapter's terms are summed in K order by the tensor core whatever
// other adapters share the tile, so a token's bits do not depend on the rest of the pass (packed rows give the bits
// of padded ones). Waits are bounded (%globaltimer, 2 s): on expiry the CTA records JB_DEV_TIMEOUT | 60.. in the
// device status word and returns. Passes of at most 128 tokens take dot_kernel (below) instead.

namespace jb {
namespace lsh {

constexpr int TM = 128;             // tokens per CTA
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int X_BYTES = TM * BK * 2;     // 16 KB
constexpr int B_BYTES = 16384;           // a stage's A rows: up to COLS rows of 128 B
constexpr int COLS = 128;                // tensor-memory columns: adapters per pass x R <= COLS
constexpr int THREADS = 192;             // warps 0-3 epilogue, 4 producer, 5 MMA
constexpr int MASK_WORDS = 8;            // a tile's adapter set as a bitmask over pool rows < 256
constexpr int MAX_POOL_ROWS = 32 * MASK_WORDS;

struct Layout {
  static constexpr int OFF_X = 0;
  static constexpr int OFF_B = OFF_X + STAGES * X_BYTES;
  static constexpr int OFF_BAR = OFF_B + STAGES * B_BYTES;
  static constexpr int NBAR = 2 * STAGES + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;        // tmem slot, abort flag, adapter count
  static constexpr int OFF_MASK = OFF_MISC + 16;
  static constexpr int OFF_LIST = OFF_MASK + MASK_WORDS * 4;   // the tile's adapters in pool-row order
  static constexpr int BYTES = OFF_LIST + TM * 4;
  static constexpr int ALLOC = BYTES + 1024;
  static_assert(ALLOC <= 227 * 1024, "shared memory");
};

// 16 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__global__ void __launch_bounds__(THREADS, 1)
    shrink_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_a, int M, int K,
                  int R, int pool_rows, const int* __restrict__ adapters, int row_len, __nv_bfloat16* __restrict__ mid,
                  int* err) {
  pdl_begin();
  using L = Layout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  int* count = reinterpret_cast<int*>(smem + L::OFF_MISC + 8);
  uint32_t* mask = reinterpret_cast<uint32_t*>(smem + L::OFF_MASK);
  int* list = reinterpret_cast<int*>(smem + L::OFF_LIST);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * TM;
  const int nkb = K / BK;
  const int per_pass = COLS / R;

  // this token's adapter (threads 0-127 are the tile's tokens); the tile's adapter set
  int my_a = 0;
  if (tid < MASK_WORDS) mask[tid] = 0;
  if (tid == 0) {
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, 4);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, COLS);
    tmem_relinquish();
  }
  __syncthreads();
  if (tid < TM && m0 + tid < M) {
    const int a = adapters[(m0 + tid) / row_len];
    my_a = (a >= 0 && a < pool_rows) ? a : 0;
    atomicOr(&mask[my_a >> 5], 1u << (my_a & 31));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    int d = 0;
    for (int w = 0; w < MASK_WORDS; ++w)
      for (uint32_t bits = mask[w]; bits; bits &= bits - 1u) list[d++] = 32 * w + __ffs(bits) - 1;
    *count = d;
  }
  __syncthreads();
  const uint32_t tmem = *tmem_slot;
  const int adapters_in_tile = *count;
  const int passes = (adapters_in_tile + per_pass - 1) / per_pass;

  if (warp == 4) {
    // ---------------- producer
    if (elect_one()) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_a);
      uint32_t it = 0;
      for (int pass = 0; pass < passes && !*abort_flag; ++pass) {
        const int first = pass * per_pass;
        const int dg = min(per_pass, adapters_in_tile - first);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, err, 60)) break;
          mbar_arrive_expect_tx(&full[s], X_BYTES + dg * R * 128);
          tma_load_2d(smem + L::OFF_X + s * X_BYTES, &tm_x, &full[s], kb * BK, m0);
          for (int j = 0; j < dg; ++j)
            tma_load_3d(smem + L::OFF_B + s * B_BYTES + j * R * 128, &tm_a, &full[s], kb * BK, 0, list[first + j]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMA issuer
    const bool issuer = elect_one();
    const uint32_t idesc = idesc_bf16(TM, R);
    uint32_t it = 0;
    bool ok = true;
    for (int pass = 0; pass < passes && ok; ++pass) {
      const int dg = min(per_pass, adapters_in_tile - pass * per_pass);
      // the epilogue has read the previous pass's columns
      ok = __all_sync(0xffffffffu, mbar_wait(tmem_empty, (pass & 1) ^ 1, abort_flag, err, 61));
      if (!ok) break;
      tc_fence_after();
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % STAGES;
        ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (it / STAGES) & 1, abort_flag, err, 62));
        if (!ok) break;
        tc_fence_after();
        const uint64_t xd = sw128_desc(smem_u32(smem + L::OFF_X + s * X_BYTES));
        const uint64_t bd = sw128_desc(smem_u32(smem + L::OFF_B + s * B_BYTES));
        if (issuer) {
          for (int j = 0; j < dg; ++j)
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              tc_mma_bf16(tmem + j * R, xd + 2 * kk, bd + (uint64_t)((j * R * 128) >> 4) + 2 * kk, idesc,
                          (kb | kk) != 0);
          tc_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (issuer) tc_commit(tmem_full);
      __syncwarp();
    }
  } else {
    // ---------------- epilogue: thread = token tid (TMEM lane tid)
    const uint32_t lane_bits = (uint32_t)(32 * warp) << 16;
    const int t = m0 + tid;
    for (int pass = 0; pass < passes; ++pass) {
      const bool ok = __all_sync(0xffffffffu, mbar_wait(tmem_full, pass & 1, abort_flag, err, 63));
      if (!ok) break;
      tc_fence_after();
      const int first = pass * per_pass;
      const int dg = min(per_pass, adapters_in_tile - first);
      for (int j = 0; j < dg; ++j) {
        const bool mine = t < M && list[first + j] == my_a;
        for (int c0 = 0; c0 < R; c0 += 16) {   // every lane joins each load; a token keeps its own adapter's
          uint32_t r[16];
          tmem_ld16(tmem + lane_bits + j * R + c0, r);
          tc_wait_ld();
          if (mine) {
            uint4 v0, v1;
            v0.x = pack_bf2(__uint_as_float(r[0]), __uint_as_float(r[1]));
            v0.y = pack_bf2(__uint_as_float(r[2]), __uint_as_float(r[3]));
            v0.z = pack_bf2(__uint_as_float(r[4]), __uint_as_float(r[5]));
            v0.w = pack_bf2(__uint_as_float(r[6]), __uint_as_float(r[7]));
            v1.x = pack_bf2(__uint_as_float(r[8]), __uint_as_float(r[9]));
            v1.y = pack_bf2(__uint_as_float(r[10]), __uint_as_float(r[11]));
            v1.z = pack_bf2(__uint_as_float(r[12]), __uint_as_float(r[13]));
            v1.w = pack_bf2(__uint_as_float(r[14]), __uint_as_float(r[15]));
            uint4* dst = reinterpret_cast<uint4*>(mid + (size_t)t * R + c0);
            dst[0] = v0;
            dst[1] = v1;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tmem_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, COLS);
  }
}

// Small passes (at most DOT_MAX_M tokens): one warp per (token, rank) dot, DOT_ROWS ranks of one token per CTA
// (grid: tokens x ceil(R / DOT_ROWS)), so a 32-token pass of rank 48 runs 384 CTAs instead of a latency chain on a
// few SMs. Each lane reads its 16-byte pieces i = lane, lane + 32, ... of the x row and of the adapter's A row (both
// from L2, several pieces in flight), sums its fp32 products in K order, then a fixed-order butterfly across the
// lanes; one bf16 rounding. Every (token, rank) is independent of the rest of the pass, so packed rows still give the
// bits of padded ones. The tcgen05 kernel streams one 128-token tile's whole K through a single CTA, which at these
// sizes is a latency chain of 16 to 56 K blocks.
constexpr int DOT_MAX_M = 128;
constexpr int DOT_THREADS = 128;
constexpr int DOT_ROWS = DOT_THREADS / 32;   // ranks per CTA: one per warp

__global__ void __launch_bounds__(DOT_THREADS) dot_kernel(const __nv_bfloat16* __restrict__ x, int K, int R,
                                                          int pool_rows, const int* __restrict__ adapters,
                                                          int row_len, const __nv_bfloat16* __restrict__ A,
                                                          __nv_bfloat16* __restrict__ mid) {
  pdl_begin();
  const int t = blockIdx.x;
  const int r = blockIdx.y * DOT_ROWS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= R) return;   // whole warps
  int a = adapters[t / row_len];
  if (a < 0 || a >= pool_rows) a = 0;   // pool row 0: the zero adapter
  const uint4* xs = reinterpret_cast<const uint4*>(x + (size_t)t * K);
  const uint4* ar = reinterpret_cast<const uint4*>(A + ((size_t)a * R + r) * K);
  float acc = 0.f;
#pragma unroll 4
  for (int i = lane; i < K / 8; i += 32) {
    const uint4 av = __ldg(ar + i), xv = __ldg(xs + i);
    acc = fmaf(bf_lo(av.x), bf_lo(xv.x), acc);
    acc = fmaf(bf_hi(av.x), bf_hi(xv.x), acc);
    acc = fmaf(bf_lo(av.y), bf_lo(xv.y), acc);
    acc = fmaf(bf_hi(av.y), bf_hi(xv.y), acc);
    acc = fmaf(bf_lo(av.z), bf_lo(xv.z), acc);
    acc = fmaf(bf_hi(av.z), bf_hi(xv.z), acc);
    acc = fmaf(bf_lo(av.w), bf_lo(xv.w), acc);
    acc = fmaf(bf_hi(av.w), bf_hi(xv.w), acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) mid[(size_t)t * R + r] = f2bf(acc);
}

// mid = bf16(x A[a]^T) for every token; JB_OK, or an error status (jb_last_error) when a map or the launch fails
int launch(const __nv_bfloat16* x, int m, int k, const __nv_bfloat16* a, int rank, int pool_rows,
           const int* adapters, int row_len, __nv_bfloat16* mid, cudaStream_t stream) {
  if (m <= DOT_MAX_M) {
    launch_pdl(dot_kernel, dim3(m, (rank + DOT_ROWS - 1) / DOT_ROWS), DOT_THREADS, 0, stream, x, k, rank, pool_rows,
                                                                                     adapters, row_len, a, mid);
    return check_launch("lora shrink dot_kernel");
  }
  CUtensorMap tx, ta;
  int st = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k, m, (uint64_t)k * 2, BK, TM,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  const uint64_t dims[3] = {(uint64_t)k, (uint64_t)rank, (uint64_t)pool_rows};
  const uint64_t strides[2] = {(uint64_t)k * 2, (uint64_t)rank * k * 2};
  const uint32_t box[3] = {BK, (uint32_t)rank, 1};
  st = make_tmap_nd(&ta, a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  cudaError_t e = cudaFuncSetAttribute(shrink_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout::ALLOC);
  if (e != cudaSuccess) return status_of(e, "lora shrink_kernel (tcgen05): shared memory attribute");
  launch_pdl(shrink_kernel, (m + TM - 1) / TM, THREADS, Layout::ALLOC, stream, tx, ta, m, k, rank, pool_rows, adapters,
                                                                       row_len, mid, device_status_word());
  return check_launch("lora shrink_kernel (tcgen05)");
}

}  // namespace lsh
}  // namespace jb
