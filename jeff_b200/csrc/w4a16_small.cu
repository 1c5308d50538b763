// S1 for small passes: the int4 W4A16 + multi-LoRA product of at most 64 tokens, streaming the weights.
//
// At a few dozen tokens the product is a stream of int4 weights (4.2 MB for the Gated DeltaNet in_proj) past a tiny
// activation block: HBM moves it in well under a microsecond, so what costs is latency. Measured on a B200, every
// hand-off of a stage ring (an mbarrier round trip between two threads of a CTA) costs 400-750 cycles whatever the
// bytes, an L2 round trip to data another SM wrote costs 1.5-2 us, and a CTA that walks a tile's whole K through a
// ring pays the first for every K block. So here:
//   - one CTA per (128-column tile, K slice), the slices of a tile one thread-block cluster (grid tiles x S,
//     cluster 1 x S); the slice's K blocks arrive by four TMA copies onto one mbarrier: the x tiles of every block
//     (a 3-D box: 64 inputs x the pass's tokens rounded up to 16 x the blocks, 128-byte swizzle), the packed words of
//     every block, and the scale and zero rows they use;
//   - two groups of four warps (thread = weight column) dequantise the blocks, alternately, into `nw` weight tiles
//     (the MMA's A, 128-byte swizzle, K-major), a batch of nw blocks at a time with one proxy fence and one barrier
//     arrival per warp; warp 1 waits once per batch and issues tcgen05.mma (M 128, N the tokens, K 16) x 4 per block
//     into a TMEM accumulator, then one commit frees the batch's tiles for the next;
//   - the LoRA expand (the pass's rows, at most two, each its adapter): per row one more K block, its B rows
//     (128 columns x rank, zeros past rank) by TMA and its tokens' mid rows (zeros for the other row's tokens) by the
//     dequantisers' own loads, issued before the base block wait; row r is added by slice r % S;
//   - the first group's threads (thread = TMEM lane) read the accumulator and store each token's fp32 sum straight
//     into the inbox of the cluster CTA that owns the token (CTA o stores tokens [o x_rows / S, (o + 1) x_rows / S)),
//     at the slot of this slice; one cluster barrier later every CTA adds its tokens' S sums from its own shared
//     memory in slice order (a fixed order: deterministic), rounds once and stores y (the SwiGLU form of the
//     persistent kernel: gate columns 0-63 of a tile, up 64-127, out = bf16(bf16(silu(g)) u)).
// Every token's sums are its own (tokens never mix), so packed rows give the bits of padded ones. Waits on mbarriers
// are bounded (%globaltimer): on expiry the CTA records JB_DEV_TIMEOUT | 70.. and skips the rest of its work; it
// still joins the cluster barrier, so the cluster ends.

namespace jb {
namespace w4s {

constexpr int BN = 128;            // weight columns per tile: the MMA's M, the TMEM lanes
constexpr int BK = 64;
constexpr int MAX_M = 64;          // tokens: the MMA's N is the pass rounded up to 16
constexpr int MAX_ROWS = 2;        // LoRA rows of a pass (one expand block each)
constexpr int MAX_NW = 4;          // dequantised weight tiles (4, or 2 where 4 do not fit)
constexpr int THREADS = 320;       // warp 0 producer, warp 1 MMA, warps 2-5 and 6-9 the two dequantiser groups
constexpr int MAX_SPLIT = 8;       // cluster size (portable)
constexpr int RAW_BYTES = 8 * BN * 4;   // 4 KB of packed words per K block
constexpr int SC_BYTES = 256;           // a scale (or zero) row of 128 bf16
constexpr int W_BYTES = BN * BK * 2;    // 16 KB
constexpr int STG_PITCH = BN + 8;       // epilogue staging: bf16 elements per token row
constexpr int TMEM_COLS = 64;
constexpr int SMEM_LIMIT = 227 * 1024;

struct Params {
  int M, K, columns, out, group;
  const __nv_bfloat16* mid;        // (M, rank) or null
  const int* adapters;
  int rank, row_len, pool_rows, rows;   // rows: LoRA rows of the pass (<= MAX_ROWS), 0 without LoRA
  int swiglu;
  int x_rows;                      // tokens rounded up to 16: the x box rows and the MMA's N
  int split, kbs, nw, ng;          // K slices per tile (cluster size), K blocks per slice, weight tiles, scale rows
  __nv_bfloat16* y;
  int ldy;
  int* err;
};

// shared-memory layout of a launch (x_rows, kbs, the expand rows, nw and the scale rows ng are per launch)
struct Layout {
  int off_raw, off_sc, off_zr, off_x, off_w, off_ex, off_ew, off_in, off_bar, off_misc, bytes;
  __host__ __device__ Layout(int x_rows, int kbs, int rows, int nw, int ng) {
    off_raw = 0;
    off_sc = off_raw + kbs * RAW_BYTES;
    off_zr = off_sc + ng * SC_BYTES;
    off_x = ((off_zr + ng * SC_BYTES + 1023) / 1024) * 1024;       // 128-byte swizzle: 1024-byte aligned
    off_w = off_x + kbs * x_rows * 128;
    off_ex = off_w + nw * W_BYTES;                                 // the expand's x slots
    off_ew = off_ex + rows * x_rows * 128;                         // ... and B tiles (1024-aligned)
    off_in = off_ew + rows * W_BYTES;                              // the inbox: [slice][column][own tokens] fp32
    off_bar = off_in + BN * x_rows * 4;
    off_misc = off_bar + (2 + 2 * MAX_NW + 2) * 8;
    bytes = off_misc + 16;
  }
};

// Phase trace (built only with -DJB_TRACE): CTAs (x < 8, y = 0) stamp %globaltimer at their phases into
// g_small_trace[event][cta]: 0 entry, 1 barriers and TMEM ready, 3 loads issued, 5 base loads landed, 6 last block
// dequantised, 7 first MMA issued, 8 last MMA committed, 9 accumulator ready, 10 sums parked, 11 slices added and
// stored, 12 before TMEM release, 13 exit; g_small_span[0 / 1][cta] every CTA's entry and exit. Without JB_TRACE the
// stamps compile to nothing.
#ifdef JB_TRACE
__device__ unsigned long long g_small_trace[14][8];
__device__ unsigned long long g_small_span[2][1024];
#define JB_SMALL(ev)                                                                        \
  do {                                                                                      \
    if (blockIdx.x < 8 && blockIdx.y == 0) g_small_trace[ev][blockIdx.x] = global_ns();     \
  } while (0)
#define JB_SPAN(ev)                                                                         \
  do {                                                                                      \
    const unsigned c = blockIdx.y * gridDim.x + blockIdx.x;                                 \
    if (c < 1024u) g_small_span[ev][c] = global_ns();                                       \
  } while (0)
#else
#define JB_SMALL(ev) \
  do {               \
  } while (0)
#define JB_SPAN(ev) \
  do {              \
  } while (0)
#endif

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// every thread of every CTA of the cluster: what each wrote to shared memory before is visible to all after
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// stores v at shared address `saddr` (16-byte aligned, this CTA's layout) of the cluster's CTA `rank`
__device__ __forceinline__ void st_peer_f32x4(uint32_t saddr, uint32_t rank, float4 v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(saddr), "r"(rank));
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

template <bool ZERO>
__global__ void __launch_bounds__(THREADS, 1)
    small_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                 const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
                 const __grid_constant__ CUtensorMap tm_lb, Params p) {
  pdl_begin();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, ks = blockIdx.y, S = p.split, NW = p.nw;
  const int n0 = tile * BN;
  // this slice's expand rows: r = ks, ks + S, ... below p.rows
  const int erows = p.rows > ks ? (p.rows - ks + S - 1) / S : 0;
  const Layout L(p.x_rows, p.kbs, p.rows, NW, p.ng);   // room for every row's expand block (one slice: them all)
  // the slices must be one cluster: a launch without it (a tool replaying the kernel without its cluster shape)
  // records JB_DEV_LAUNCH and touches no other CTA's shared memory
  uint32_t nctarank;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(nctarank));
  const bool clustered = nctarank == (uint32_t)S;
  const int XB = p.x_rows * 128;
  const int tpc = p.x_rows / S;                   // tokens each CTA of the cluster stores, a multiple of 4
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.off_bar);   // the slice's base loads
  uint64_t* efull = full + 1;                                        // the expand's B tiles
  uint64_t* dq = efull + 1;                                          // a batch of weight tiles (and x slots) ready
  uint64_t* wf = dq + 1;                                             // a batch's MMAs completed: its tiles free
  uint64_t* tmem_full = wf + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.off_misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.off_misc + 4);
  volatile int* flag = reinterpret_cast<volatile int*>(smem + L.off_misc + 8);
  if (tid == 0) {
    JB_SMALL(0);
    JB_SPAN(0);
    mbar_init(full, 1);
    mbar_init(efull, 1);
    mbar_init(dq, 8);   // the eight dequantiser warps
    mbar_init(wf, 1);
    mbar_init(tmem_full, 1);
    *abort_flag = clustered ? 0 : 1;
    *flag = 0;
    if (!clustered && p.err) atomicCAS(p.err, 0, JB_DEV_LAUNCH | 70);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) JB_SMALL(1);
  const int kb0 = ks * p.kbs;
  const int g_lo = (kb0 * BK) / p.group;   // the first scale row of the slice

  if (warp == 0) {
    // ---------------- producer: every load of the slice at once
    if (elect_one()) {
      mbar_arrive_expect_tx(full, (uint32_t)(p.kbs * (XB + RAW_BYTES) + p.ng * SC_BYTES * (ZERO ? 2 : 1)));
      tma_load_3d(smem + L.off_x, &tm_x, full, 0, 0, kb0);
      tma_load_2d(smem + L.off_raw, &tm_w, full, n0, kb0 * (BK / 8));
      tma_load_2d(smem + L.off_sc, &tm_s, full, n0, g_lo);
      if (ZERO) tma_load_2d(smem + L.off_zr, &tm_z, full, n0, g_lo);
      if (erows) {
        // each expand row's B rows for this tile (rows past the pool's, for an invalid adapter: zeros)
        mbar_arrive_expect_tx(efull, (uint32_t)erows * W_BYTES);
        for (int e = 0; e < erows; ++e) {
          const int a = p.adapters[ks + e * S];
          const int brow = (a >= 0 && a < p.pool_rows) ? a * p.columns + n0 : p.pool_rows * p.columns;
          tma_load_2d(smem + L.off_ew + e * W_BYTES, &tm_lb, efull, 0, brow);
        }
      }
      JB_SMALL(3);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (the warp computes the uniform descriptors; one elected lane issues)
    const bool issuer = elect_one();
    const uint32_t idesc = idesc_bf16(BN, p.x_rows);
    bool ok = true;
    for (int b0 = 0, u = 0; b0 < p.kbs && ok; b0 += NW, ++u) {
      ok = __all_sync(0xffffffffu, mbar_wait(dq, u & 1, abort_flag, p.err, 71));
      if (!ok) break;
      tc_fence_after();
      const int b1 = min(p.kbs, b0 + NW);
      for (int j = b0; j < b1; ++j) {
        const uint64_t ad = sw128_desc(smem_u32(smem + L.off_w + (j - b0) * W_BYTES));
        const uint64_t bd = sw128_desc(smem_u32(smem + L.off_x + j * XB));
        if (issuer) {
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) tc_mma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (j | kk) != 0);
        }
      }
      if (issuer) {
        if (b1 < p.kbs) tc_commit(wf);
        if (u == 0) JB_SMALL(7);
      }
      __syncwarp();
    }
    if (ok && erows) {
      // the expand: B tiles by TMA (efull), x slots with the last batch (dq); rank / 16 MMAs per row
      ok = __all_sync(0xffffffffu, mbar_wait(efull, 0, abort_flag, p.err, 75));
      if (ok) {
        tc_fence_after();
        for (int e = 0; e < erows; ++e) {
          const uint64_t ad = sw128_desc(smem_u32(smem + L.off_ew + e * W_BYTES));
          const uint64_t bd = sw128_desc(smem_u32(smem + L.off_ex + e * XB));
          if (issuer)
            for (int kk = 0; kk < p.rank / 16; ++kk) tc_mma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, 1);
        }
      }
    }
    if (issuer) {
      tc_commit(tmem_full);
      JB_SMALL(8);
    }
    __syncwarp();
  } else {
    // ---------------- dequantisers: group grp (warps 2-5 or 6-9) takes the blocks j with j % 2 == grp; thread =
    // weight column n (for the first group also its TMEM lane, which the epilogue reads)
    const int grp = (warp - 2) >> 2;
    const int et = tid - 64 - 128 * grp;
    const int n = 32 * (warp & 3) + lane;
    // the expand's mid pieces of token row n, requested before the base loads land (first group only)
    uint4 mv[8];
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) mv[c8] = make_uint4(0, 0, 0, 0);
    const int my_row = n < p.M ? n / p.row_len : -1;
    const bool my_expand = grp == 0 && erows > 0 && my_row >= 0 && my_row < p.rows && my_row % S == ks;
    if (my_expand) {
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        if (8 * c8 < p.rank) mv[c8] = *reinterpret_cast<const uint4*>(p.mid + (size_t)n * p.rank + 8 * c8);
    }
    bool ok = mbar_wait(full, 0, abort_flag, p.err, 72);
    if (et == 0 && grp == 0) JB_SMALL(5);
    // batches of NW blocks: each group dequantises its blocks of the batch (the first group, in the last batch, also
    // the expand's x slots), then one fence and one arrival per warp
    for (int b0 = 0, u = 0; b0 < p.kbs; b0 += NW, ++u) {
      if (u > 0) ok = ok && mbar_wait(wf, (u - 1) & 1, abort_flag, p.err, 73);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      const int b1 = min(p.kbs, b0 + NW);
      for (int j = b0 + grp; j < b1; j += 2) {
        uint8_t* wt = smem + L.off_w + (j - b0) * W_BYTES;
        const int gr = ((kb0 + j) * BK) / p.group - g_lo;
        const int32_t* raw = reinterpret_cast<const int32_t*>(smem + L.off_raw + j * RAW_BYTES);
        const __nv_bfloat16* sc = reinterpret_cast<const __nv_bfloat16*>(smem + L.off_sc + gr * SC_BYTES);
        const __nv_bfloat16* zr =
            ZERO ? reinterpret_cast<const __nv_bfloat16*>(smem + L.off_zr + gr * SC_BYTES) : nullptr;
        const __nv_bfloat162 s2 = __bfloat162bfloat162(sc[n]);
        const __nv_bfloat162 zb2 = w4::zero_pair(zr, n);
        uint32_t wd[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) wd[r] = static_cast<uint32_t>(raw[r * BN + n]);
#pragma unroll
        for (int r = 0; r < 8; ++r)
          *reinterpret_cast<uint4*>(wt + sw128_offset(n, r)) = w4::dequant8(wd[r], s2, zb2);
      }
      if (b1 == p.kbs && grp == 0 && erows && n < p.x_rows) {
        // x slot e: the mid rows of expand row ks + e S's tokens, zeros for every other token
        for (int e = 0; e < erows; ++e) {
          const bool mine = my_expand && my_row == ks + e * S;
          uint8_t* xt = smem + L.off_ex + e * XB;
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8)
            *reinterpret_cast<uint4*>(xt + sw128_offset(n, c8)) = mine ? mv[c8] : make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq);
    }
    if (et == 0 && grp == 0) JB_SMALL(6);
    if (grp == 0) {
      // the accumulator: each token's fp32 sum into the inbox of the CTA that owns it, at this slice's slot
      if (et == 0) *flag = (clustered && ok && mbar_wait(tmem_full, 0, abort_flag, p.err, 74)) ? 1 : 0;
      named_barrier(1, 128);
      if (et == 0) JB_SMALL(9);
      if (*flag) {
        tc_fence_after();
        const uint32_t acc = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        const uint32_t inbox = smem_u32(smem + L.off_in) + (uint32_t)((ks * BN + n) * tpc) * 4u;
#pragma unroll 1
        for (int t0 = 0; t0 < p.x_rows; t0 += 16) {
          uint32_t r[16];
          tmem_ld16(acc + t0, r);
          tc_wait_ld();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int t = t0 + 4 * q, owner = t / tpc;
            st_peer_f32x4(inbox + (uint32_t)(t - owner * tpc) * 4u, (uint32_t)owner,
                          make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                      __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])));
          }
        }
      }
      if (et == 0) JB_SMALL(10);
    }
  }

  // every CTA of the cluster has stored its sums (or given up): add this CTA's tokens, S slots each, in slice order
  __syncthreads();
  cluster_sync_all();
  if (warp >= 2 && warp < 6) {
    const int et = tid - 64;
    const int n = 32 * (warp & 3) + lane;
    const int t_lo = ks * tpc;
    __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem + L.off_w);   // staging: tpc tokens x 128 columns
    const float* in = reinterpret_cast<const float*>(smem + L.off_in);
    const int ow = p.swiglu ? p.out / 2 : p.out;
    if (*flag) {
#pragma unroll 1
      for (int t = 0; t < tpc; t += 4) {
        float4 v = *reinterpret_cast<const float4*>(in + n * tpc + t);
#pragma unroll 1
        for (int s = 1; s < S; ++s) {
          const float4 u = *reinterpret_cast<const float4*>(in + (s * BN + n) * tpc + t);
          v.x += u.x;
          v.y += u.y;
          v.z += u.z;
          v.w += u.w;
        }
        stg[(t + 0) * STG_PITCH + n] = f2bf(v.x);
        stg[(t + 1) * STG_PITCH + n] = f2bf(v.y);
        stg[(t + 2) * STG_PITCH + n] = f2bf(v.z);
        stg[(t + 3) * STG_PITCH + n] = f2bf(v.w);
      }
      named_barrier(1, 128);
      if (!p.swiglu) {
        for (int i = et; i < tpc * (BN / 8); i += 128) {
          const int tt = i / (BN / 8), c8 = i % (BN / 8);
          const int gm = t_lo + tt, col = n0 + 8 * c8;
          if (gm < p.M && col < ow)
            *reinterpret_cast<uint4*>(p.y + (size_t)gm * p.ldy + col) =
                *reinterpret_cast<const uint4*>(stg + tt * STG_PITCH + 8 * c8);
        }
      } else {
        // columns 0-63 of the tile are gate, 64-127 the matching up columns: 64 outputs bf16(bf16(silu(g)) u)
        for (int i = et; i < tpc * (BN / 16); i += 128) {
          const int tt = i / (BN / 16), c8 = i % (BN / 16);
          const int gm = t_lo + tt, col = n0 / 2 + 8 * c8;
          if (gm < p.M && col < ow) {
            const uint4 gv = *reinterpret_cast<const uint4*>(stg + tt * STG_PITCH + 8 * c8);
            const uint4 uv = *reinterpret_cast<const uint4*>(stg + tt * STG_PITCH + BN / 2 + 8 * c8);
            const uint32_t* gw = &gv.x;
            const uint32_t* uw = &uv.x;
            uint32_t ov[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              ov[e] = pack_bf2(w4::silu_rounded(bf_lo(gw[e])) * bf_lo(uw[e]),
                               w4::silu_rounded(bf_hi(gw[e])) * bf_hi(uw[e]));
            *reinterpret_cast<uint4*>(p.y + (size_t)gm * p.ldy + col) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
          }
        }
      }
    }
    if (et == 0) JB_SMALL(11);
  }
  __syncthreads();
  if (tid == 0) {
    JB_SMALL(12);
    if (*abort_flag) {
      // a wait gave up: let this CTA's copies still in flight land before it exits (bounded)
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(full, 0) && global_ns() - t0 < kWaitNs) {
      }
      while (erows && !mbar_try_wait(efull, 0) && global_ns() - t0 < 2 * kWaitNs) {
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
    if (lane == 0) {
      JB_SMALL(13);
      JB_SPAN(1);
    }
  }
}

// scale (or zero) rows a slice of kbs K blocks can touch
inline int scale_rows(int kbs, int group) { return (kbs * BK + group - 1) / group + 1; }
// shared-memory bytes of a launch (with its alignment slack)
inline int smem_bytes(int x_rows, int kbs, int rows, int nw, int group) {
  return Layout(x_rows, kbs, rows, nw, scale_rows(kbs, group)).bytes + 1024;
}
// the weight tiles a slice of kbs blocks gets: 4 (at most kbs) where they fit, else 2 (0: neither fits)
inline int choose_nw(int x_rows, int kbs, int rows, int group) {
  if (kbs > 32) return 0;   // the words box: 8 kbs rows <= 256
  for (int nw = kbs < MAX_NW ? (kbs < 2 ? 2 : kbs) : MAX_NW; nw >= 2; nw -= 2)
    if (smem_bytes(x_rows, kbs, rows, nw, group) <= SMEM_LIMIT) return nw;
  return 0;
}

// K slices for a pass of `tiles` column tiles and `kb` K blocks: among 1, 2, 4 and 8 dividing kb (and leaving each
// CTA a multiple of 4 tokens to store) whose slice fits in shared memory (one CTA per SM), the most whose grid
// still fits on the SMs at once, else the fewest (0: none fits)
inline int choose_split(int tiles, int kb, int x_rows, int rows, int group, int sms) {
  int best = 0;
  for (int s = 1; s <= MAX_SPLIT; s *= 2) {
    if (kb % s || (x_rows / s) % 4 || !choose_nw(x_rows, kb / s, rows, group)) continue;
    if (best == 0 || tiles * s <= sms) best = s;
  }
  return best;
}

// the K slices the small-pass kernel would run a pass with (0: it does not take the pass)
inline int plan(int m, int k, int columns, int rank, int row_len, int group) {
  if (m < 1 || m > MAX_M || k % BK || row_len <= 0 || (group != 64 && group != 128)) return 0;
  const int rows = rank > 0 ? (m + row_len - 1) / row_len : 0;
  if (rows > MAX_ROWS) return 0;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return choose_split((columns + BN - 1) / BN, k / BK, ((m + 15) / 16) * 16, rows, group, sms);
}

// the small-pass product (m <= MAX_M, LoRA rows <= MAX_ROWS); split 0 chooses the K slices, otherwise split must be
// 1, 2, 4 or 8, divide k / 64 and leave a slice that fits in shared memory
static int launch(const uint16_t* x, int m, int k, const int32_t* words, const uint16_t* scales,
                  const uint16_t* zeros, int group, int columns, int out, const uint16_t* mid, const uint16_t* lora_b,
                  int rank, int pool_rows, const int32_t* adapters, int row_len, uint16_t* y, int ldy, bool swiglu,
                  int split, cudaStream_t stream) {
  const int x_rows = ((m + 15) / 16) * 16;
  const int tiles = (columns + BN - 1) / BN;
  const int kb = k / BK;
  const bool lora = mid != nullptr && rank > 0;
  const int rows = lora ? (m + row_len - 1) / row_len : 0;
  JB_REQUIRE(m >= 1 && m <= MAX_M, "small product: m %d (1 to %d)", m, MAX_M);
  JB_REQUIRE(rows <= MAX_ROWS, "small product: %d LoRA rows (at most %d)", rows, MAX_ROWS);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (split <= 0) split = choose_split(tiles, kb, x_rows, rows, group, sms);
  JB_REQUIRE(split >= 1 && split <= MAX_SPLIT && (split & (split - 1)) == 0 && kb % split == 0 &&
                 (x_rows / split) % 4 == 0,
             "small product: %d K slices for %d K blocks and %d token rows (1, 2, 4 or 8 dividing the blocks, "
             "leaving a multiple of 4 tokens per slice)", split, kb, x_rows);
  const int kbs = kb / split;
  const int nw = choose_nw(x_rows, kbs, rows, group);
  JB_REQUIRE(nw > 0, "small product: a slice of %d K blocks needs %d bytes of shared memory", kbs,
             smem_bytes(x_rows, kbs, rows, 2, group));
  const int smem = smem_bytes(x_rows, kbs, rows, nw, group);
  const int ng = scale_rows(kbs, group);
  CUtensorMap tx, tw, ts, tz, tl;
  int st;
  {
    // x as (64 inputs, m tokens, k / 64 blocks): one box of every block of a slice, block-major in shared memory
    const uint64_t dims[3] = {(uint64_t)BK, (uint64_t)m, (uint64_t)kb};
    const uint64_t strides[2] = {(uint64_t)k * 2, (uint64_t)BK * 2};
    const uint32_t box[3] = {BK, (uint32_t)x_rows, (uint32_t)kbs};
    if ((st = make_tmap_nd(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  }
  if ((st = make_tmap_2d(&tw, words, CU_TENSOR_MAP_DATA_TYPE_INT32, columns, k / 8, (uint64_t)columns * 4, BN,
                         8 * kbs, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return st;
  if ((st = make_tmap_2d(&ts, scales, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, columns, k / group, (uint64_t)columns * 2,
                         BN, ng, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return st;
  if (zeros) {
    if ((st = make_tmap_2d(&tz, zeros, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, columns, k / group, (uint64_t)columns * 2,
                           BN, ng, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return st;
  } else {
    tz = ts;
  }
  if (lora) {
    // B rows (pool_rows x columns, rank): a 64-wide box of 128 rows, zeros past rank, in the 128-byte swizzle
    if ((st = make_tmap_2d(&tl, lora_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, (uint64_t)pool_rows * columns,
                           (uint64_t)rank * 2, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  } else {
    tl = ts;
  }
  Params p{m, k, columns, out, group, lora ? reinterpret_cast<const __nv_bfloat16*>(mid) : nullptr, adapters,
           lora ? rank : 0, row_len > 0 ? row_len : 1, pool_rows, rows, swiglu ? 1 : 0, x_rows, split, kbs, nw, ng,
           reinterpret_cast<__nv_bfloat16*>(y), ldy, device_status_word()};
  auto kern = zeros ? small_kernel<true> : small_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return status_of(e, "small product: shared memory attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, split);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = split;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, kern, tx, tw, ts, tz, tl, p);
  if (e != cudaSuccess) return status_of(e, "w4a16 small_kernel launch");
  return check_launch("w4a16 small_kernel");
}

}  // namespace w4s
}  // namespace jb
