// S3 on tcgen05: paged prefix-KV gated attention with S and O in tensor memory, K / V pages by TMA, and the output
// gate fused into the epilogue.
//
// One CTA per (row, key/value head g, 32 new tokens). Its 128 query rows are the 32 tokens x the 4 query heads that
// share head g (row 32 h + i: query head 4 g + h, token 32 qb + i), the Q tile (128 x 256 bf16) loaded once by TMA.
// Keys are walked in tiles of 64: the prefix's pool pages two at a time (the page of token j is tables[r][kv_entry +
// j / 32]), then the row's own new keys up to the block's last token. Per tile:
//   S = Q K^T      tcgen05.mma M 128, N 64, K 256 (16 steps) into one of two S buffers in tensor memory;
//   softmax        8 warps, thread = half a query row (its tensor-memory lane): masks (prefix keys past the prefix length,
//                  new keys after the row's own token), the running max in log2 units, P = exp2(s - m) rounded to
//                  bf16 (the reference's rounding point, batched_kernels.py:405-427) written to shared memory in the
//                  MMA's 128B-swizzled layout, the row sum from the unrounded values; V rows of keys past the prefix
//                  (stale page contents) are zeroed before the value product reads them;
//   O += P V       tcgen05.mma M 128, N 256, K 64 (4 steps), O fp32 in tensor memory (256 columns), V as an
//                  MN-major operand straight from its pages.
// The softmax keeps O's scale until the running max has grown by more than 8 (a factor 256): only then it waits for
// the previous value product and rescales O in tensor memory. The epilogue divides by the row sum, rounds O to bf16,
// multiplies by bf16(sigmoid(gate)) (the gate half of the row's q_proj output) and rounds again: the reference's
// gate_mul (fast_path.py:123-138), written straight into the o_proj input y (t, 2048).
// Warps: 0 TMA producer, 1 tensor-memory allocation + MMA issue (one thread), 2-9 softmax and epilogue (two warps per
// row: each takes half of a tile's scores and half of O's columns; the halves' maxima meet in shared memory). Every wait
// is bounded (2 s of %globaltimer): a lost arrival ends the kernel with a device status instead of a hang.

namespace jb {
namespace atc {

constexpr int NQ = 8, NKV = 2, HD = 256, PAGE = 32;
constexpr int BQ = 32;                 // new tokens per CTA (x 4 heads = 128 query rows)
constexpr int BKN = 64;                // keys per tile
constexpr int STAGES = 2;              // K / V tile ring
constexpr int Q_BYTES = 128 * HD * 2;            // 64 KB: 4 chunks of 64 dims x 128 rows x 128 B
constexpr int KV_BYTES = BKN * HD * 2;           // 32 KB per K or V tile: 4 chunks of 64 dims x 64 keys x 128 B
constexpr int P_BYTES = 128 * BKN * 2;           // 16 KB
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_BYTES;
constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
constexpr int OFF_P = OFF_V + STAGES * KV_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
// barriers: q_full, k_full[2], v_full[2], k_free[2], v_free[2], s_full[2], p_ready[2], o_done[2], xchg[2], xsum
constexpr int NBAR = 2 + 8 * STAGES;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int OFF_RED = OFF_MISC + 16;           // softmax exchange: maxima [2 tiles][2 halves][128 rows] (fp32)
constexpr int SMEM = OFF_RED + 4 * 128 * 4;
// the swizzled tiles need a 1024-byte aligned base; the dynamic shared memory of a kernel with no static shared
// memory starts there, which the kernel checks (and reports through the status word instead of running misaligned)
constexpr int ALLOC = SMEM;
static_assert(ALLOC <= 227 * 1024, "shared memory");
constexpr int TM_S = 0;                // S buffer b at column TM_S + 64 b
constexpr int TM_O = 256;              // O at columns [256, 512)
constexpr int THREADS = 10 * 32;

struct Params {
  const int* tables;
  int table_stride, kv_entry, attn_layer, attn_layers;
  const int* pos;
  const __nv_bfloat16* pr;   // the q_proj | k | v output: the gate of head h at column 512 h + 256
  int ldpr;
  __nv_bfloat16* y;
  int ldy;
  int n;
  float scale_log2;
  int* err;
  // split walk: gridDim.z slices of each row's key tiles; slice z writes its unnormalised O, running max and row sum
  // to part (O [z][token][query head][256], then m, l [z][token][query head][2], fp32) and combine_kernel finishes
  int splits;
  float* part;
};

// 2^x by the hardware's approximate base-2 exponential (PTX ex2.approx.ftz.f32), as the reference's Triton
// tl.exp2 does; -inf and very negative arguments give +0
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// K-major SW128 descriptor (rows of 128 B, 8-row groups 1024 B apart), as common.cuh's sw128_desc
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) { return sw128_desc(saddr); }
// MN-major SW128 descriptor: rows (K direction) of 128 B = 64 N elements, 8-row groups SBO = 1024 B apart along K,
// 64-element N atoms LBO bytes apart
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t saddr, uint32_t lbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__global__ void __launch_bounds__(THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_pool,
                     const __grid_constant__ CUtensorMap tm_kn, const __grid_constant__ CUtensorMap tm_vn, Params p) {
  pdl_begin();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if (smem_u32(smem) & 1023u) {   // uniform over the CTA: every thread returns before any barrier or allocation
    if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, JB_DEV_TIMEOUT | 99);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* k_free = v_full + STAGES;     // a K tile is free once its Q K^T is done, a V tile once its P V is
  uint64_t* v_free = k_free + STAGES;
  uint64_t* s_full = v_free + STAGES;
  uint64_t* p_ready = s_full + 2;
  uint64_t* o_done = p_ready + 2;
  uint64_t* xchg = o_done + 2;           // the 8 softmax warps' row maxima of tile j are in (by tile parity)
  uint64_t* xsum_bar = xchg + 2;         // their row sums are in
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  const int row = blockIdx.x / NKV, g = blockIdx.x % NKV;
  const int qb = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = p.pos[row];
  const int pre_tiles = (P + BKN - 1) / BKN;
  const int q_hi = (qb + 1) * BQ;                      // new keys this block may see: [0, q_hi)
  const int all_tiles = pre_tiles + (q_hi + BKN - 1) / BKN;
  // this CTA's key tiles [j0, j0 + tiles) of the row's, an even slice when the walk is split; barrier phases count
  // the CTA's own tiles (jj), key positions the row's (j)
  const int j0 = (int)((long long)all_tiles * blockIdx.z / p.splits);
  const int tiles = (int)((long long)all_tiles * (blockIdx.z + 1) / p.splits) - j0;
  const int tok0 = row * p.n + qb * BQ;                 // the block's first token in the pass

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_free[s], 1);
      mbar_init(&v_free[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[s], 8);
      mbar_init(&o_done[s], 1);
      mbar_init(&xchg[s], 8);
    }
    mbar_init(xsum_bar, 8);
    *abort_flag = 0;
    fence_barrier_init();
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
    // ---------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_pool);
      prefetch_tmap(&tm_kn);
      prefetch_tmap(&tm_vn);
      mbar_arrive_expect_tx(q_full, Q_BYTES);
      for (int h = 0; h < 4; ++h)
        for (int c = 0; c < 4; ++c)
          tma_load_3d(smem + OFF_Q + c * (128 * 128) + h * (BQ * 128), &tm_q, q_full, 64 * c, 4 * g + h,
                      tok0);
      // the source rows of tile j's two 32-key halves: pool rows of the prefix pages (a page past the prefix's last
      // reads the sink page: masked, its V rows zeroed), or rows of the new keys
      auto load = [&](int j, bool values, uint8_t* dst, uint64_t* bar) {
        for (int half = 0; half < 2; ++half) {
          int r0;
          const CUtensorMap* map;
          if (j < pre_tiles) {
            const int pi = 2 * j + half;
            const int page = pi * PAGE < P ? p.tables[(size_t)row * p.table_stride + p.kv_entry + pi] : 0;
            r0 = ((page * p.attn_layers + p.attn_layer) * 2 + (values ? 1 : 0)) * PAGE;
            map = &tm_pool;
          } else {
            r0 = row * p.n + (j - pre_tiles) * BKN + half * PAGE;
            map = values ? &tm_vn : &tm_kn;
          }
          for (int c = 0; c < 4; ++c) tma_load_3d(dst + c * (BKN * 128) + half * (PAGE * 128), map, bar, 64 * c, g, r0);
        }
      };
      for (int jj = 0; jj < tiles; ++jj) {
        const int s = jj % STAGES;
        const uint32_t ph = ((jj / STAGES) & 1) ^ 1;
        if (!mbar_wait(&k_free[s], ph, abort_flag, p.err, 21)) break;
        mbar_arrive_expect_tx(&k_full[s], KV_BYTES);
        load(j0 + jj, false, smem + OFF_K + s * KV_BYTES, &k_full[s]);
        if (!mbar_wait(&v_free[s], ph, abort_flag, p.err, 31)) break;
        mbar_arrive_expect_tx(&v_full[s], KV_BYTES);
        load(j0 + jj, true, smem + OFF_V + s * KV_BYTES, &v_full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: S_0, S_1, PV_0, S_2, PV_1, ... (the next tile's Q K^T runs during a softmax)
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(128, BKN);
      constexpr uint32_t idesc_o = idesc_bf16(128, HD) | (1u << 16);   // B (V) MN-major
      const uint32_t qa = smem_u32(smem + OFF_Q);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err, 22);
      auto issue_s = [&](int j) -> bool {
        const int s = j % STAGES;
        if (!mbar_wait(&k_full[s], (j / STAGES) & 1, abort_flag, p.err, 23)) return false;
        // S buffer j % 2 is free once the softmax of tile j - 2 is done with it (its p_ready)
        if (j >= 2 && !mbar_wait(&p_ready[j & 1], ((j - 2) >> 1) & 1, abort_flag, p.err, 24)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(smem + OFF_K + s * KV_BYTES);
        const uint32_t d = tmem + TM_S + 64 * (j & 1);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int c = kk >> 2, w = kk & 3;
          tc_mma_bf16(d, kmajor_desc(qa + c * (128 * 128) + 32 * w), kmajor_desc(ka + c * (BKN * 128) + 32 * w),
                      idesc_s, kk != 0);
        }
        tc_commit(&s_full[j & 1]);
        tc_commit(&k_free[s]);
        return true;
      };
      auto issue_o = [&](int j) -> bool {
        const int s = j % STAGES;
        if (!mbar_wait(&v_full[s], (j / STAGES) & 1, abort_flag, p.err, 30)) return false;
        if (!mbar_wait(&p_ready[j & 1], (j >> 1) & 1, abort_flag, p.err, 25)) return false;
        tc_fence_after();
        const uint32_t pa = smem_u32(smem + OFF_P + (j & 1) * P_BYTES);
        const uint32_t va = smem_u32(smem + OFF_V + s * KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKN / 16; ++kk)
          tc_mma_bf16(tmem + TM_O, kmajor_desc(pa + 32 * kk), mnmajor_desc(va + kk * 16 * 128, BKN * 128), idesc_o,
                      (j | kk) != 0);
        tc_commit(&v_free[s]);
        tc_commit(&o_done[j & 1]);
        return true;
      };
      if (ok && tiles > 0) ok = issue_s(0);
      for (int j = 0; ok && j < tiles; ++j) {
        if (j + 1 < tiles) ok = issue_s(j + 1);
        if (ok) ok = issue_o(j);
      }
    }
  } else {
    // ---------------- softmax + epilogue: 8 warps, two per tensor-memory lane quadrant. Thread = query row r = 32 h
    // + i (its lane) and one half of the row's scores (keys [32 half, + 32) of each tile) and of its O columns
    // ([128 half, + 128)); the two halves' maxima meet through shared memory, their sums at the end.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = 32 * quad + lane;
    const int h = r >> 5, i = r & 31;
    const int tok = qb * BQ + i;                       // this row's new-token index within its row of the pass
    const uint32_t lane_bits = (uint32_t)(32 * quad) << 16;
    float* xmax = reinterpret_cast<float*>(smem + OFF_RED);          // [2 tiles][2 halves][128 rows]
    float m = -1e30f, l = 0.f;
    bool ok = true;
    for (int jj = 0; jj < tiles && ok; ++jj) {
      const int j = j0 + jj;
      ok = mbar_wait(&s_full[jj & 1], (jj >> 1) & 1, abort_flag, p.err, 26);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      uint32_t sv[32];   // this half's 32 scores of the row
      tmem_ld32(tmem + lane_bits + TM_S + 64 * (jj & 1) + 32 * half, sv);
      tc_wait_ld();
      const bool prefix = j < pre_tiles;
      const int key0 = (prefix ? j * BKN : (j - pre_tiles) * BKN) + 32 * half;
      const int limit = prefix ? P - key0 : tok + 1 - key0;   // keys [key0, key0 + limit) of this half are valid
      float mine = -1e30f;   // the max of the raw scores; scaled below (scale_log2 > 0 keeps the order)
#pragma unroll
      for (int c = 0; c < 32; ++c)
        if (c < limit) mine = fmaxf(mine, __uint_as_float(sv[c]));
      mine = mine > -1e30f ? mine * p.scale_log2 : -1e30f;
      xmax[((jj & 1) * 2 + half) * 128 + r] = mine;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xchg[jj & 1]);
      ok = mbar_wait(&xchg[jj & 1], (jj >> 1) & 1, abort_flag, p.err, 32);   // both halves' maxima of tile j are in
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      const float mx = fmaxf(m, fmaxf(mine, xmax[((jj & 1) * 2 + (half ^ 1)) * 128 + r]));
      // P buffer j % 2 is free once the value product of tile j - 2 is done (o_done); O may be rescaled only after
      // the value product of tile j - 1
      if (jj >= 1) {
        const bool rescale = mx > m + 8.0f;
        // warp-uniform: a warp that rescales any of its rows touches all 32 rows' O, so it waits for tile j - 1
        const int wait_for = __any_sync(0xffffffffu, rescale) ? jj - 1 : jj - 2;
        if (wait_for >= 0) {
          ok = mbar_wait(&o_done[wait_for & 1], (wait_for >> 1) & 1, abort_flag, p.err, 27);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, rescale)) {   // tensor-memory loads are warp-wide: the warp rescales together
          const float alpha = rescale ? ex2(m - mx) : 1.0f;
#pragma unroll 1
          for (int cc = 0; cc < HD / 64; ++cc) {   // this half's 128 O columns
            uint32_t ov[32];
            const uint32_t oa = tmem + lane_bits + TM_O + 128 * half + 32 * cc;
            tmem_ld32(oa, ov);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            w4t::tmem_st32(oa, ov);
          }
          w4t::tc_wait_st();
          l *= alpha;
          if (rescale) m = mx;
        }
      } else {
        m = mx;
      }
      // P = bf16(exp2(s - m)) into the swizzled K-major P tile (row r: 64 keys = 128 B; this half's 4 chunks of 16
      // B), this half's row sum unrounded
      uint8_t* pt = smem + OFF_P + (jj & 1) * P_BYTES;
      float rs = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        float e8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = 8 * c8 + e;
          e8[e] = c < limit ? ex2(fmaf(__uint_as_float(sv[c]), p.scale_log2, -m)) : 0.f;
          rs += e8[e];
        }
        *reinterpret_cast<uint4*>(pt + sw128_offset(r, 4 * half + c8)) =
            make_uint4(pack_bf2(e8[0], e8[1]), pack_bf2(e8[2], e8[3]), pack_bf2(e8[4], e8[5]), pack_bf2(e8[6], e8[7]));
      }
      l += rs;
      const int tile_key0 = prefix ? j * BKN : 0;
      if (prefix && P - tile_key0 < BKN) {
        // stale page contents past the prefix: zero those V rows (P is 0 there, but 0 x NaN is NaN)
        const int s = jj % STAGES;
        ok = mbar_wait(&v_full[s], (jj / STAGES) & 1, abort_flag, p.err, 28);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        uint8_t* vt = smem + OFF_V + s * KV_BYTES;
        const int first = P - tile_key0 > 0 ? P - tile_key0 : 0;
        for (int idx = threadIdx.x - 64; idx < (BKN - first) * 4 * 8; idx += 256) {   // rows x 4 chunks x 8 x 16 B
          const int key = first + idx / 32, rest = idx % 32, c = rest / 8, piece = rest % 8;
          *reinterpret_cast<uint4*>(vt + c * (BKN * 128) + key * 128 + piece * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[jj & 1]);
    }
    // ---------------- epilogue: O / l -> bf16, times bf16(sigmoid(gate)) -> y (this half's 128 columns). The two
    // halves' sums meet in the exchange buffer of the parity the last tile did not use (its last reader, tile
    // tiles - 2, finished before the last tile's barrier).
    float* xsum = xmax + (tiles & 1) * 2 * 128;   // (tiles: this CTA's own count)
    xsum[half * 128 + r] = l;
    __syncwarp();
    if (lane == 0) mbar_arrive(xsum_bar);
    ok = ok && mbar_wait(xsum_bar, 0, abort_flag, p.err, 33);
    l += xsum[(half ^ 1) * 128 + r];
    if (ok && tiles > 0) {
      const int jl = tiles - 1;
      ok = mbar_wait(&o_done[jl & 1], (jl >> 1) & 1, abort_flag, p.err, 29);
    }
    if (__all_sync(0xffffffffu, ok) && p.splits > 1) {
      // a slice of a split walk: unnormalised O (relative to this slice's max m), m and l for combine_kernel
      tc_fence_after();
      const int t = tok0 + i;
      const int qh = 4 * g + h;
      const size_t tq = ((size_t)blockIdx.z * gridDim.x / NKV * p.n + t) * NQ + qh;   // (slice, token, head)
      float* orow = p.part + tq * HD + 128 * half;
#pragma unroll 1
      for (int cc = 0; cc < HD / 64; ++cc) {
        uint32_t ov[32];
        if (tiles > 0) {
          tmem_ld32(tmem + lane_bits + TM_O + 128 * half + 32 * cc, ov);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = 0u;
        }
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          *reinterpret_cast<float4*>(orow + 32 * cc + 4 * q4) =
              make_float4(__uint_as_float(ov[4 * q4]), __uint_as_float(ov[4 * q4 + 1]),
                          __uint_as_float(ov[4 * q4 + 2]), __uint_as_float(ov[4 * q4 + 3]));
      }
      if (half == 0) {
        float* ml = p.part + (size_t)p.splits * (gridDim.x / NKV) * p.n * NQ * HD + tq * 2;
        ml[0] = m;
        ml[1] = l;
      }
    } else if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      const int t = tok0 + i;
      const int qh = 4 * g + h;
      const __nv_bfloat16* gate = p.pr + (size_t)t * p.ldpr + qh * 2 * HD + HD + 128 * half;
      __nv_bfloat16* yrow = p.y + (size_t)t * p.ldy + qh * HD + 128 * half;
#pragma unroll 1
      for (int cc = 0; cc < HD / 64; ++cc) {
        uint32_t ov[32];
        tmem_ld32(tmem + lane_bits + TM_O + 128 * half + 32 * cc, ov);
        tc_wait_ld();
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const uint4 gv = *reinterpret_cast<const uint4*>(gate + 32 * cc + 8 * q8);
          const float g8[8] = {bf_lo(gv.x), bf_hi(gv.x), bf_lo(gv.y), bf_hi(gv.y),
                               bf_lo(gv.z), bf_hi(gv.z), bf_lo(gv.w), bf_hi(gv.w)};
          float o8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float o = round_bf(__uint_as_float(ov[8 * q8 + e]) * inv);
            o8[e] = o * round_bf(1.0f / (1.0f + expf(-g8[e])));
          }
          *reinterpret_cast<uint4*>(yrow + 32 * cc + 8 * q8) =
              make_uint4(pack_bf2(o8[0], o8[1]), pack_bf2(o8[2], o8[3]), pack_bf2(o8[4], o8[5]),
                         pack_bf2(o8[6], o8[7]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// The slices of a split walk, per (token, query head): M = the slices' largest max, O = sum_z 2^(m_z - M) O_z,
// L = sum_z 2^(m_z - M) l_z in slice order (deterministic); then the unsplit epilogue: bf16(O / L) times
// bf16(sigmoid(gate)), rounded. One block of 256 threads (one per value column) per (token, query head).
__global__ void __launch_bounds__(HD) combine_kernel(const float* __restrict__ part, int splits, int tokens,
                                                     const __nv_bfloat16* __restrict__ pr, int ldpr,
                                                     __nv_bfloat16* __restrict__ y, int ldy) {
  pdl_begin();
  const int t = blockIdx.x / NQ, qh = blockIdx.x % NQ, d = threadIdx.x;
  const size_t rows = (size_t)tokens * NQ;
  const float* ml = part + (size_t)splits * rows * HD;
  float M = -1e30f;
  for (int z = 0; z < splits; ++z) M = fmaxf(M, ml[(z * rows + blockIdx.x) * 2]);
  float o = 0.f, L = 0.f;
  for (int z = 0; z < splits; ++z) {
    const float mz = ml[(z * rows + blockIdx.x) * 2], lz = ml[(z * rows + blockIdx.x) * 2 + 1];
    const float w = lz > 0.f ? ex2(mz - M) : 0.f;
    o += w * part[(z * rows + blockIdx.x) * HD + d];
    L += w * lz;
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  const float g = bf2f(pr[(size_t)t * ldpr + qh * 2 * HD + HD + d]);
  y[(size_t)t * ldy + qh * HD + d] = f2bf(round_bf(o * inv) * round_bf(1.0f / (1.0f + expf(-g))));
}

// A 3-D bf16 tensor map {HD dims, heads, rows} with head stride `head_bytes` and row stride `row_bytes`, box
// {64 dims, 1 head, 32 rows}, 128-byte swizzle: one load lands 32 rows x 128 B in the MMA's swizzled layout.
inline int make_map(CUtensorMap* map, const void* base, uint64_t heads, uint64_t rows, uint64_t head_bytes,
                    uint64_t row_bytes) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (head_bytes & 15) || (row_bytes & 15)) {
    set_error("attention tensor map: base %p, strides %llu / %llu must be 16-byte aligned", base,
              (unsigned long long)head_bytes, (unsigned long long)row_bytes);
    return JB_EINVAL;
  }
  cudaDriverEntryPointQueryResult q;
  void* fnp = nullptr;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fnp, 12000, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fnp) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return JB_ECUDA;
  }
  auto fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fnp);
  cuuint64_t dims[3] = {(cuuint64_t)HD, heads, rows};
  cuuint64_t strides[2] = {head_bytes, row_bytes};
  cuuint32_t box[3] = {64, 1, 32};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (attention) failed (%d): %llu heads x %llu rows", (int)r,
              (unsigned long long)heads, (unsigned long long)rows);
    return JB_ECUDA;
  }
  return JB_OK;
}

}  // namespace atc
}  // namespace jb

namespace jb {
namespace atc {
// the gated attention with the key walk in `splits` slices (1: the whole walk in one CTA, no scratch)
static int gated_impl(const uint16_t* q, const void* pool, int64_t pool_pages, int64_t page_bytes,
                      const int32_t* tables, int table_stride, int kv_entry, int attn_layer, int attn_layers,
                      const int32_t* pos, const uint16_t* kn, const uint16_t* vn, const uint16_t* pr, int ldpr,
                      uint16_t* y, int ldy, int b, int n, int splits, float* part, void* stream) {
  JB_REQUIRE(q && pool && tables && pos && kn && vn && pr && y, "jb_paged_attention_gated: null pointer");
  JB_REQUIRE(b > 0 && n > 0 && n % atc::BQ == 0, "jb_paged_attention_gated: b %d, n %d (a multiple of 32)", b, n);
  JB_REQUIRE(pool_pages > 0 && attn_layer >= 0 && attn_layer < attn_layers &&
                 (int64_t)attn_layers * 2 * atc::PAGE * atc::NKV * atc::HD * 2 == page_bytes,
             "jb_paged_attention_gated: attention layer %d of %d in pages of %lld bytes (the pages must hold exactly "
             "the keys and values of every attention layer)", attn_layer, attn_layers, (long long)page_bytes);
  JB_REQUIRE(kv_entry >= 0 && kv_entry <= table_stride, "jb_paged_attention_gated: kv_entry %d", kv_entry);
  JB_REQUIRE(ldpr >= atc::NQ * 2 * atc::HD && ldpr % 8 == 0 && ldy >= atc::NQ * atc::HD && ldy % 8 == 0,
             "jb_paged_attention_gated: ldpr %d, ldy %d", ldpr, ldy);
  JB_REQUIRE(((reinterpret_cast<uintptr_t>(pr) | reinterpret_cast<uintptr_t>(y)) & 15) == 0,
             "jb_paged_attention_gated: pr and y must be 16-byte aligned");
  CUtensorMap tq, tpool, tkn, tvn;
  const uint64_t t = (uint64_t)b * n;
  int st;
  if ((st = atc::make_map(&tq, q, atc::NQ, t, atc::HD * 2, (uint64_t)atc::NQ * atc::HD * 2))) return st;
  if ((st = atc::make_map(&tpool, pool, atc::NKV, (uint64_t)pool_pages * attn_layers * 2 * atc::PAGE, atc::HD * 2,
                          (uint64_t)atc::NKV * atc::HD * 2)))
    return st;
  if ((st = atc::make_map(&tkn, kn, atc::NKV, t, atc::HD * 2, (uint64_t)atc::NKV * atc::HD * 2))) return st;
  if ((st = atc::make_map(&tvn, vn, atc::NKV, t, atc::HD * 2, (uint64_t)atc::NKV * atc::HD * 2))) return st;
  atc::Params p{tables, table_stride, kv_entry, attn_layer, attn_layers, pos,
                reinterpret_cast<const __nv_bfloat16*>(pr), ldpr, reinterpret_cast<__nv_bfloat16*>(y), ldy, n,
                (1.0f / 16.0f) * 1.4426950408889634f, device_status_word(), splits, part};
  if ((st = status_of(cudaFuncSetAttribute(atc::attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           atc::ALLOC), "attention: shared memory attribute")))
    return st;
  dim3 grid(b * atc::NKV, n / atc::BQ, splits);
  launch_pdl(atc::attention_kernel, grid, atc::THREADS, atc::ALLOC, (cudaStream_t)stream, tq, tpool, tkn, tvn, p);
  if ((st = check_launch("attention_kernel (tcgen05)"))) return st;
  if (splits > 1) {
    launch_pdl(atc::combine_kernel, (unsigned)(t * atc::NQ), atc::HD, 0, (cudaStream_t)stream,
        part, splits, (int)t, reinterpret_cast<const __nv_bfloat16*>(pr), ldpr, reinterpret_cast<__nv_bfloat16*>(y),
        ldy);
    return check_launch("attention combine_kernel");
  }
  return JB_OK;
}
}  // namespace atc
}  // namespace jb

extern "C" int jb_paged_attention_gated(const uint16_t* q, const void* pool, int64_t pool_pages, int64_t page_bytes,
                                        const int32_t* tables, int table_stride, int kv_entry, int attn_layer,
                                        int attn_layers, const int32_t* pos, const uint16_t* kn, const uint16_t* vn,
                                        const uint16_t* pr, int ldpr, uint16_t* y, int ldy, int b, int n,
                                        void* stream) {
  return jb::atc::gated_impl(q, pool, pool_pages, page_bytes, tables, table_stride, kv_entry, attn_layer,
                             attn_layers, pos, kn, vn, pr, ldpr, y, ldy, b, n, 1, nullptr, stream);
}

extern "C" int jb_paged_attention_gated_split(const uint16_t* q, const void* pool, int64_t pool_pages,
                                              int64_t page_bytes, const int32_t* tables, int table_stride,
                                              int kv_entry, int attn_layer, int attn_layers, const int32_t* pos,
                                              const uint16_t* kn, const uint16_t* vn, const uint16_t* pr, int ldpr,
                                              uint16_t* y, int ldy, int b, int n, float* scratch,
                                              int64_t scratch_floats, void* stream) {
  using namespace jb;
  JB_REQUIRE(scratch && (reinterpret_cast<uintptr_t>(scratch) & 15) == 0,
             "jb_paged_attention_gated_split: scratch must be a 16-byte aligned pointer");
  JB_REQUIRE(b > 0 && n > 0 && n % atc::BQ == 0, "jb_paged_attention_gated_split: b %d, n %d (a multiple of 32)",
             b, n);
  // slices only when the CTAs of the unsplit walk leave SMs idle: enough slices to cover the SMs (at most 16), as
  // many as the scratch holds (per slice, O and m, l of every token and query head)
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ctas = b * atc::NKV * (n / atc::BQ);
  const int64_t per_slice = (int64_t)b * n * atc::NQ * (atc::HD + 2);
  int splits = ctas >= sms ? 1 : (sms + ctas - 1) / ctas;
  if (splits > 16) splits = 16;
  while (splits > 1 && splits * per_slice > scratch_floats) --splits;
  return atc::gated_impl(q, pool, pool_pages, page_bytes, tables, table_stride, kv_entry, attn_layer, attn_layers,
                         pos, kn, vn, pr, ldpr, y, ldy, b, n, splits, scratch, stream);
}
