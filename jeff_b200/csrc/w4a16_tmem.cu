// S1, tensor-memory form: the int4 W4A16 product with the dequantised weights as the tensor core's A operand in
// tensor memory (swapped roles: D^T = W . x^T), tcgen05 + TMA (sm_100a), persistent.
//
// Why: in the shared-memory form (w4a16_gemm.cu) every K block moves the x tile in by TMA, the dequantised weight
// tile out of the dequantisers and both operands into the tensor core, all through shared memory; at the tensor
// rate that traffic is above what shared memory delivers, so the MMAs wait on it. Here the dequantisers write the
// weight tile straight from registers into tensor memory (tcgen05.st), where the MMA reads it as A; shared memory
// carries only the x tile (TMA in, tensor core out) and the packed words: about a third fewer bytes per FLOP.
//
// Tile: 128 weight columns (MMA M, tensor-memory lanes) x 256 tokens (MMA N), K blocks of 64, fp32 accumulator
// D[column][token] in tensor memory (one accumulator beside the A ring; the producer and the dequantisers run ahead
// into the next tile while the epilogue drains it), tiles token-tile major so concurrent CTAs share one x tile and
// walk the (smaller) int4 weights through L2. Each dequantised weight serves 256 tokens. Warps:
//   warp 0       TMA producer: per K block the x tile (256 tokens x 64, 128B swizzle), the packed words (8 x 128
//                int32) and the group's scale (and zero) row, into a STAGES-deep ring (mbarrier full[s]);
//   warp 1       allocates 512 tensor-memory columns ([0, 256) the accumulator, [256, 256 + 32 STAGES) the A
//                ring: 32 columns = 128 lanes x 64 bf16 per stage); one thread issues tcgen05.mma (M 128, N 256,
//                K 16, A from tensor memory, B = the x tile) x 4 per K block after ONE wait (deq[s]: the
//                dequantisers arrive only after they saw full[s], so it covers the x tile too);
//   warps 2-9    two warpgroups on alternate K blocks; thread = weight column (its tensor-memory lane): 8 words ->
//                64 bf16 = bf16((u - z) s) -> tcgen05.st of 32 columns into the stage's A slot (deq[s]);
//   warps 10-13  epilogue: tcgen05.ld of 32 tokens per load -> bf16 -> y[token][column] (lane-consecutive columns:
//                one 64-byte row piece per warp store), or with `swiglu` the gate lanes (0-63) take their up lane's
//                value (64 above) through shared memory and write bf16(bf16(silu(g)) u).
// LoRA (rows of a multiple of 128 tokens: one adapter per 128-token half): one extra K block of depth rank per half:
// the producer loads the half's mid rows (128 tokens x rank, planes of 8 columns) by TMA as B, the dequantisers load
// their column's rank values of the half's adapter's B row into the A slot, and an N = 128 MMA adds it into the
// half's accumulator columns.
// One rounding at the end. Every output is the same fp32 sum in the same K order as the shared-memory form.

namespace jb {
namespace w4t {

constexpr int BM = 128;              // weight columns per tile
constexpr int BT = 256;              // tokens per tile (one N = 256 MMA per K16 step)
constexpr int HT = 128;              // tokens per LoRA half (one adapter per 128 tokens)
constexpr int BK = 64;
constexpr int STAGES = 5;
constexpr int GROUPS = 2;
constexpr int DEQ_WARPS = 8;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 64 + (DEQ_WARPS + EPI_WARPS) * 32;
constexpr int NACC = 512 - STAGES * (BK / 2) >= 2 * BT ? 2 : 1;   // accumulators that fit beside the A ring
constexpr int TM_ACC = 0;            // tensor-memory column of accumulator b: TM_ACC + b * BT
constexpr int TM_A = NACC * BT;      // tensor-memory column of A slot s: TM_A + s * (BK / 2)
static_assert(TM_A + STAGES * (BK / 2) <= 512, "tensor memory");

struct Params {
  int M, K, columns, out, group;
  const __nv_bfloat16* lora_b;       // (pool_rows, columns, rank) or null
  const int* adapters;
  int rank, row_len, pool_rows;
  int swiglu;
  int t_tiles, n_tiles;
  __nv_bfloat16* y;
  int ldy;
  int* err;
  int planes3d;
};

struct Layout {
  static constexpr int X_BYTES = BT * BK * 2;      // 32 KB
  static constexpr int RAW_BYTES = 8 * BM * 4;     // 4 KB
  static constexpr int SC_BYTES = BM * 2;
  static constexpr int OFF_X = 0;
  static constexpr int OFF_RAW = OFF_X + STAGES * X_BYTES;
  static constexpr int OFF_SC = OFF_RAW + STAGES * RAW_BYTES;
  static constexpr int OFF_ZR = OFF_SC + STAGES * SC_BYTES;
  static constexpr int OFF_BAR = OFF_ZR + STAGES * SC_BYTES;
  static constexpr int NBAR = 3 * STAGES + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_ADP = OFF_MISC + 16;
  static constexpr int MAX_ROWS = 512;
  static constexpr int OFF_SWAP = OFF_ADP + MAX_ROWS * 4;   // SwiGLU: the up values of 32 tokens x 64 columns
  static constexpr int BYTES = OFF_SWAP + 32 * 64 * 4;
  static constexpr int ALLOC = BYTES + 1024;
  static_assert(ALLOC <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <bool ZERO>
__global__ void __launch_bounds__(THREADS, 1)
    w4a16_tmem_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                      const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
                      const __grid_constant__ CUtensorMap tm_mid, Params p) {
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
  int* s_adp = reinterpret_cast<int*>(smem + L::OFF_ADP);
  float* swap = reinterpret_cast<float*>(smem + L::OFF_SWAP);   // [32 tokens][64 columns]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nkb = p.K / BK;
  const bool has_lora = p.lora_b != nullptr && p.rank > 0;
  const int tiles = p.t_tiles * p.n_tiles;
  if (has_lora) {
    const int rows = (p.M + p.row_len - 1) / p.row_len;
    for (int i = threadIdx.x; i < rows && i < L::MAX_ROWS; i += blockDim.x) {
      const int a = p.adapters[i];
      s_adp[i] = (a >= 0 && a < p.pool_rows) ? a : -1;
    }
  }
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
    if (has_lora) prefetch_tmap(&tm_mid);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkt = nkb + (has_lora ? BT / HT : 0);   // the base K blocks, then one LoRA block per 128-token half

  if (warp == 0) {
    // ---------------- producer
    if (lane == 0) {
      const uint32_t bytes = L::X_BYTES + L::RAW_BYTES + L::SC_BYTES * (ZERO ? 2 : 1);
      const int planes = p.rank / 8;
      uint32_t kg = 0;
      for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
        const int t0 = (tile / p.n_tiles) * BT, n0 = (tile % p.n_tiles) * BM;
        for (int kb = 0; kb < nkt; ++kb, ++kg) {
          const int s = kg % STAGES;
          if (!mbar_wait(&empty[s], ((kg / STAGES) & 1) ^ 1, abort_flag, p.err, 11)) break;
          uint8_t* xs = smem + L::OFF_X + s * L::X_BYTES;
          if (kb < nkb) {
            mbar_arrive_expect_tx(&full[s], bytes);
            tma_load_2d(xs, &tm_x, &full[s], kb * BK, t0);
            tma_load_2d(smem + L::OFF_RAW + s * L::RAW_BYTES, &tm_w, &full[s], n0, kb * (BK / 8));
            tma_load_2d(smem + L::OFF_SC + s * L::SC_BYTES, &tm_s, &full[s], n0, (kb * BK) / p.group);
            if (ZERO) tma_load_2d(smem + L::OFF_ZR + s * L::SC_BYTES, &tm_z, &full[s], n0, (kb * BK) / p.group);
          } else {
            // LoRA block of half h: its mid rows (rank / 8 planes of 128 rows x 16 B; rows past m read zeros)
            const int r0 = t0 + (kb - nkb) * HT;
            mbar_arrive_expect_tx(&full[s], planes * 2048);
            if (p.planes3d) {
              tma_load_3d(xs, &tm_mid, &full[s], 0, r0, 0);
            } else {
              for (int c = 0; c < planes; ++c) tma_load_2d(xs + c * 2048, &tm_mid, &full[s], 8 * c, r0);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BT);
      constexpr uint32_t idesc_half = idesc_bf16(BM, HT);
      uint32_t kg = 0;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++it) {
        const int b = it % NACC;
        ok = mbar_wait(&tmem_empty[b], ((it / NACC) & 1) ^ 1, abort_flag, p.err, 12);
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + TM_ACC + b * BT;
        for (int kb = 0; kb < nkt; ++kb, ++kg) {
          const int s = kg % STAGES;
          ok = mbar_wait(&deq[s], (kg / STAGES) & 1, abort_flag, p.err, 13);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_tm = tmem + TM_A + s * (BK / 2);
          const uint32_t xa = smem_u32(smem + L::OFF_X + s * L::X_BYTES);
          if (kb < nkb) {
            const uint64_t bd = sw128_desc(xa);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) tc_mma_ts(acc, a_tm + 8 * kk, bd + 2 * kk, idesc, (kb | kk) != 0);
          } else {
            const uint32_t acc_h = acc + (kb - nkb) * HT;   // this half's 128 token columns
            for (int j = 0; j < p.rank / 16; ++j)
              tc_mma_ts(acc_h, a_tm + 8 * j, planes_desc(xa + 2 * j * 2048, 2048), idesc_half, 1);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&tmem_full[b]);
      }
    }
  } else if (warp < 2 + DEQ_WARPS) {
    // ---------------- dequantisers: group g on the K blocks with kg % 2 == g; thread = weight column n (its lane)
    const int grp = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int n = 32 * quad + lane;
    const uint32_t lane_bits = (uint32_t)(32 * quad) << 16;
    uint32_t kg = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
      const int t0 = (tile / p.n_tiles) * BT, n0 = (tile % p.n_tiles) * BM;
      for (int kb = 0; kb < nkt; ++kb, ++kg) {
        if ((int)(kg % GROUPS) != grp) continue;
        const int s = kg % STAGES;
        ok = mbar_wait(&full[s], (kg / STAGES) & 1, abort_flag, p.err, 14);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_tm = tmem + lane_bits + TM_A + s * (BK / 2);
        uint32_t v[32];
        if (kb < nkb) {
          const int32_t* raw = reinterpret_cast<const int32_t*>(smem + L::OFF_RAW + s * L::RAW_BYTES);
          const __nv_bfloat16* sc = reinterpret_cast<const __nv_bfloat16*>(smem + L::OFF_SC + s * L::SC_BYTES);
          const __nv_bfloat16* zr =
              ZERO ? reinterpret_cast<const __nv_bfloat16*>(smem + L::OFF_ZR + s * L::SC_BYTES) : nullptr;
          const __nv_bfloat162 s2 = __bfloat162bfloat162(sc[n]);
          const __nv_bfloat162 zb2 = w4::zero_pair(zr, n);
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const uint4 q = w4::dequant8(static_cast<uint32_t>(raw[r * BM + n]), s2, zb2);
            v[4 * r + 0] = q.x;
            v[4 * r + 1] = q.y;
            v[4 * r + 2] = q.z;
            v[4 * r + 3] = q.w;
          }
          tmem_st32(a_tm, v);
        } else {
          // the adapter's B row of this column: rank bf16 values (zeros for an invalid adapter or a padding column)
          const int r0 = t0 + (kb - nkb) * HT;
          const int a = r0 < p.M ? s_adp[r0 / p.row_len] : -1;
          const int gn = n0 + n;
          const bool live = a >= 0 && gn < p.columns;
          const uint4* src = reinterpret_cast<const uint4*>(p.lora_b + ((size_t)(live ? a : 0) * p.columns +
                                                                        (live ? gn : 0)) * p.rank);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 q = (live && c < p.rank / 8) ? src[c] : make_uint4(0, 0, 0, 0);
            v[4 * c + 0] = q.x;
            v[4 * c + 1] = q.y;
            v[4 * c + 2] = q.z;
            v[4 * c + 3] = q.w;
          }
#pragma unroll
          for (int c = 0; c < 4; ++c)   // rank / 16 stores of 8 columns (uniform over the warp)
            if (c < p.rank / 16) tmem_st8(a_tm + 8 * c, v + 8 * c);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&deq[s]);
      }
    }
  } else {
    // ---------------- epilogue: thread = weight column n (its lane); 32 tokens per tensor-memory load
    const int et = threadIdx.x - 64 - DEQ_WARPS * 32;
    const int quad = warp & 3;
    const int n = 32 * quad + lane;
    const uint32_t lane_bits = (uint32_t)(32 * quad) << 16;
    int it = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
      const int t0 = (tile / p.n_tiles) * BT, n0 = (tile % p.n_tiles) * BM;
      const int b = it % NACC;
      if (et == 0) *epi_ok = mbar_wait(&tmem_full[b], (it / NACC) & 1, abort_flag, p.err, 15) ? 1 : 0;
      named_barrier(2, EPI_WARPS * 32);
      if (!*epi_ok) break;
      tc_fence_after();
      const uint32_t acc = tmem + lane_bits + TM_ACC + b * BT;
      if (!p.swiglu) {
        const int col = n0 + n;
#pragma unroll 1
        for (int c = 0; c < BT / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(acc + c * 32, r);
          tc_wait_ld();
          if (col < p.out) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int tok = t0 + c * 32 + i;
              if (tok < p.M) p.y[(size_t)tok * p.ldy + col] = __float2bfloat16_rn(__uint_as_float(r[i]));
            }
          }
        }
      } else {
        // gate column n (lanes 0-63) and its up column n + 64 (lanes 64-127) of the tile's 64 outputs
        const int col = n0 / 2 + n;
#pragma unroll 1
        for (int c = 0; c < BT / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(acc + c * 32, r);
          tc_wait_ld();
          if (quad >= 2) {
#pragma unroll
            for (int i = 0; i < 32; ++i) swap[i * 64 + (n - 64)] = __uint_as_float(r[i]);
          }
          named_barrier(3, EPI_WARPS * 32);
          if (quad < 2 && col < p.out / 2) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int tok = t0 + c * 32 + i;
              const float g = round_bf(__uint_as_float(r[i]));
              const float u = round_bf(swap[i * 64 + n]);
              if (tok < p.M) p.y[(size_t)tok * p.ldy + col] = __float2bfloat16_rn(w4::silu_rounded(g) * u);
            }
          }
          named_barrier(3, EPI_WARPS * 32);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace w4t
}  // namespace jb

namespace jb {
namespace w4t {

// Launch on `stream`: tensor maps for x (box 64 x 128 tokens, 128B swizzle), the packed words, the scales (and
// zeros) and the mid planes; a persistent grid of min(tiles, SMs) CTAs.
inline int launch(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                  const uint16_t* zeros, int group, int columns, int out, const uint16_t* mid,
                  const uint16_t* lora_b, int rank, int pool_rows, const int32_t* adapters, int row_len, uint16_t* y,
                  int ldy, bool swiglu, cudaStream_t stream) {
  const bool lora = mid != nullptr && rank > 0;
  CUtensorMap tx, tw, ts, tz, tm;
  int st;
  if ((st = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k, m, (uint64_t)k * 2, BK, BT,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tmap_2d(&tw, words, CU_TENSOR_MAP_DATA_TYPE_INT32, columns, k / 8, (uint64_t)columns * 4, BM, 8,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
    return st;
  if ((st = make_tmap_2d(&ts, scales, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, columns, k / group, (uint64_t)columns * 2,
                         BM, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return st;
  if (zeros) {
    if ((st = make_tmap_2d(&tz, zeros, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, columns, k / group, (uint64_t)columns * 2,
                           BM, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
  } else {
    tz = ts;
  }
  int planes3d = 0;
  if (lora) {
    planes3d = make_tmap_planes(&tm, mid, m, rank, (uint64_t)rank * 2, HT) == JB_OK;
    if (!planes3d && (st = make_tmap_2d(&tm, mid, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, m, (uint64_t)rank * 2, 8,
                                        HT, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
  } else {
    tm = tx;
  }
  Params p{m, k, columns, out, group, lora ? reinterpret_cast<const __nv_bfloat16*>(lora_b) : nullptr, adapters,
           lora ? rank : 0, row_len > 0 ? row_len : BT, pool_rows, swiglu ? 1 : 0, (m + BT - 1) / BT,
           (columns + BM - 1) / BM, reinterpret_cast<__nv_bfloat16*>(y), ldy, device_status_word(), planes3d};
  int dev = 0, sms = 0;
  if ((st = status_of(cudaGetDevice(&dev), "w4a16 tmem: device"))) return st;
  if ((st = status_of(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "w4a16 tmem: SM count")))
    return st;
  const int tiles = p.t_tiles * p.n_tiles;
  const int grid = tiles < sms ? tiles : sms;
  if (zeros) {
    if ((st = status_of(cudaFuncSetAttribute(w4a16_tmem_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Layout::ALLOC), "w4a16 tmem: shared memory attribute")))
      return st;
    launch_pdl(w4a16_tmem_kernel<true>, grid, THREADS, Layout::ALLOC, stream, tx, tw, ts, tz, tm, p);
  } else {
    if ((st = status_of(cudaFuncSetAttribute(w4a16_tmem_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Layout::ALLOC), "w4a16 tmem: shared memory attribute")))
      return st;
    launch_pdl(w4a16_tmem_kernel<false>, grid, THREADS, Layout::ALLOC, stream, tx, tw, ts, tz, tm, p);
  }
  return check_launch("w4a16_tmem_kernel");
}

}  // namespace w4t
}  // namespace jb
