// S2 on tcgen05: the gated delta rule over 64-token chunks with every chunk product on the 5th-generation tensor
// cores, the fp32 state resident in tensor memory, each (row, head) resuming from its state in the prefix pool (the
// chunked form of fla's chunk_gated_delta_rule, which the reference's batched path calls at batched_path.py:282-288,
// :322-324, and of transformers' torch_chunk_gated_delta_rule on its standard path).
//
// Per chunk of C = 64 tokens (gc = cumulative log-decay within the chunk, Γ_ij = exp(gc_i - gc_j)), the same
// quantities and bf16 rounding points as the mma.sync form in gdn_chunk.cu:
//   A = strictly lower part of -diag(β) K K^T ∘ Γ, T = (I - A)^-1 (fp32 on the CUDA cores)
//   W = T (β e^gc K), U = T (β V), V' = U - W S, O = scale ((e^gc Q) S + (Q K^T ∘ Γ, causal) V'),
//   S <- e^{gc_last} S + (e^{gc_last - gc} K)^T V'.
// Tensor memory (256 columns; 128 lanes): S (key lanes x 128 value columns, fp32) in columns 0-127, D1 in 128-191,
// D2 in 192-255. The products are M = 128 tcgen05 MMAs, transposed where that puts 128 rows on the lanes:
//   MMA1  D1 = [K; Q] K^T            (lanes 0-63: K K^T rows, 64-127: Q K^T rows; the stacked A is the K and Q
//                                     tiles laid out back to back)
//   MMA2  D1 = (β e^gc K)^T T^T = W^T,  D2 = (β V)^T T^T = U^T
//   MMA3  D2 += S^T (-W^T)          -> V'^T
//   MMA4  D1 = S^T (e^gc Q)^T + V'^T P^T = O^T
//   MMA5  S += (e^{gc_last - gc} K)^T V'   (S scaled by e^{gc_last} in tensor memory beforehand)
// Warp 1 issues the MMAs (one elected lane; the warp computes the descriptors), warp 0's first lane the TMA copies:
// the chunk's K, Q and V tiles (64 tokens x 128 channels, two 64-column 128-byte-swizzled boxes each, zeros past the
// row's end) as soon as their slots are free (K after MMA2, Q and V after MMA4/5), and the chunk's output tile. The
// eight warps read each result out of tensor memory (warp w: lanes 32 (w % 4) .., columns half w / 4) and write the
// next operands into shared memory in the swizzled layouts the MMAs read (K-major or MN-major). T is solved on the
// CUDA cores: the four diagonal 16 x 16 blocks by substitution, then two doubling steps (32 x 32, then 64 x 64:
// T_21 = T_22 A_21 T_11). One CTA of 8 warps per (row, head) with about 108 KB of shared memory and 256
// tensor-memory columns, so two CTAs share an SM. The waits (MMA completion, TMA arrival) are bounded (%globaltimer,
// 2 s): on expiry the CTA records JB_DEV_TIMEOUT | 40.. in the device status word and returns.

namespace jb {
namespace gdnt {

using gdnc::C;
using gdnc::D;
using gdnc::NH;
using gdnc::PF;
using gdnc::STATE_BYTES;

constexpr int THREADS = 256;
// shared memory (offsets from a 1024-byte aligned base)
constexpr int OFF_KQ = 0;          // K | Q raw tiles per 64-column atom (atom a: K at a * 16384, Q at + 8192); then
                                   // β e^gc K over K and e^gc Q over Q
constexpr int OFF_KD = 32768;      // e^{gc_last - gc} K (atoms 8192 apart)
constexpr int OFF_V = 49152;       // V raw -> β V -> -W^T (128 key rows x 64 tokens) -> V'^T (128 value rows)
constexpr int OFF_P = 65536;       // P = Q K^T ∘ Γ causal, 64 rows x 64 (K-major)
constexpr int OFF_R = 73728;       // A and T fp32 for the solve -> T bf16 -> S bf16 (2 atoms x 128 key rows) ->
                                   // the output tile (2 atoms x 64 tokens, as the loads)
constexpr int R_BYTES = 2 * C * PF * 4;
constexpr int OFF_G = OFF_R + R_BYTES;   // gc, e^gc, e^{gc_last - gc}, β (64 floats each)
constexpr int OFF_MISC = OFF_G + 4 * C * 4;
constexpr int BYTES = OFF_MISC + 64;
constexpr int ALLOC = BYTES + 1024;
constexpr uint32_t TILE_BYTES = C * D * 2;   // one 64 x 128 bf16 tile (two 8 KB boxes)
static_assert(2 * D * 128 <= R_BYTES, "S bf16 fits the solve region");
static_assert(2 * ALLOC + 2048 <= 228 * 1024, "two CTAs per SM");

constexpr uint32_t TM_S = 0, TM_D1 = 128, TM_D2 = 192;

__device__ __forceinline__ uint64_t mn_desc(uint32_t saddr, uint32_t lbo) {
  // MN-major operand, 128-byte swizzle: rows along K of 128 B (64 M/N elements), 8-row groups 1024 B apart (SBO),
  // 64-element M/N atoms `lbo` bytes apart
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
constexpr uint32_t A_MN = 1u << 15, B_MN = 1u << 16;

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
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// e^x for x <= 0 by the hardware's base-2 exponential (ex2.approx, relative error about 2^-22): the decay factors
// inside a chunk, which the kernel then rounds to bf16 or carries into the fp32 solve
__device__ __forceinline__ float exp_neg(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
  return y;
}

// 16-byte chunk c (0..7) of row r of a 128-byte-row swizzled tile
__device__ __forceinline__ uint8_t* swz(uint8_t* tile, int r, int c) { return tile + sw128_offset(r, c); }

__device__ __forceinline__ uint4 scale8(uint4 x, float f) {
  uint4 y;
  y.x = pack_bf2(bf_lo(x.x) * f, bf_hi(x.x) * f);
  y.y = pack_bf2(bf_lo(x.y) * f, bf_hi(x.y) * f);
  y.z = pack_bf2(bf_lo(x.z) * f, bf_hi(x.z) * f);
  y.w = pack_bf2(bf_lo(x.w) * f, bf_hi(x.w) * f);
  return y;
}

__global__ void __launch_bounds__(THREADS, 2)
    scan_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                const float* __restrict__ g, const __nv_bfloat16* __restrict__ beta, int n,
                uint8_t* __restrict__ pool, int64_t page_bytes, const int* __restrict__ tables, int table_stride,
                int first_head, int heads_per_page, const int* __restrict__ last, const int* __restrict__ out_tables,
                int out_table_stride, int* err) {
  pdl_begin();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kq = sm + OFF_KQ;
  uint8_t* kd = sm + OFF_KD;
  uint8_t* vb = sm + OFF_V;
  uint8_t* pt = sm + OFF_P;
  uint8_t* rg = sm + OFF_R;
  float* amat = reinterpret_cast<float*>(rg);
  float* tf = reinterpret_cast<float*>(rg + C * PF * 4);
  float* gc = reinterpret_cast<float*>(sm + OFF_G);
  float* eg = gc + C;
  float* ed = eg + C;
  float* bt = ed + C;
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(sm + OFF_MISC);
  uint64_t* k_bar = mma_bar + 1;      // the chunk's K tile landed
  uint64_t* qv_bar = mma_bar + 2;     // its Q and V tiles landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_MISC + 24);
  volatile int* ok_flag = reinterpret_cast<volatile int*>(sm + OFF_MISC + 28);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + OFF_MISC + 32);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, ch = warp >> 2;
  const int L = 32 * qd + lane;                  // this thread's tensor-memory lane
  const uint32_t lane_bits = (uint32_t)(32 * qd) << 16;
  const int row = blockIdx.x / NH, h = blockIdx.x % NH;
  const int flat = first_head + h;
  const float scale = rsqrtf((float)D);
  const int stop = last ? min(last[row] + 1, n) : n;   // outputs past stop are written as zeros
  const size_t rbase = (size_t)row * n;
  const bool loader = tid == 0;                 // issues the TMA copies

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    mbar_init(k_bar, 1);
    mbar_init(qv_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  // the chunk at c0's tiles: K into the K slots, Q into the Q slots, V into its own (box coordinates: channel, head,
  // token of the row, row)
  int k_issued = 0, qv_issued = 0;   // loads issued (the loader's count), to drain them on the error path
  auto load_k = [&](int c0) {
    ++k_issued;
    mbar_arrive_expect_tx(k_bar, TILE_BYTES);
    tma_load_4d(kq, &tm_k, k_bar, 0, h, c0, row);
    tma_load_4d(kq + 16384, &tm_k, k_bar, 64, h, c0, row);
  };
  auto load_qv = [&](int c0) {
    ++qv_issued;
    mbar_arrive_expect_tx(qv_bar, 2 * TILE_BYTES);
    tma_load_4d(kq + 8192, &tm_q, qv_bar, 0, h, c0, row);
    tma_load_4d(kq + 16384 + 8192, &tm_q, qv_bar, 64, h, c0, row);
    tma_load_4d(vb, &tm_v, qv_bar, 0, h, c0, row);
    tma_load_4d(vb + 8192, &tm_v, qv_bar, 64, h, c0, row);
  };
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (loader) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_o);
    load_k(0);
    load_qv(0);
  }
  const uint32_t tmem = *tmem_slot;
  // gates of the next chunk, held in registers until it starts
  float g_next = 0.f, b_next = 0.f;
  if (tid < C) {
    const bool valid = tid < n;
    g_next = valid ? g[(rbase + tid) * NH + h] : 0.f;
    b_next = valid ? __bfloat162float(beta[(rbase + tid) * NH + h]) : 0.f;
  }

  // the state of this (row, head) from its pool page into tensor memory: lane = key row, columns = value; every
  // load of the thread in flight before the first store
  {
    const int page = tables[(size_t)row * table_stride + flat / heads_per_page];
    const float* s_in =
        reinterpret_cast<const float*>(pool + (int64_t)page * page_bytes + (flat % heads_per_page) * STATE_BYTES);
    const float4* src = reinterpret_cast<const float4*>(s_in + (size_t)L * D + ch * 64);
    float4 f[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) f[i] = src[i];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        r[4 * i] = __float_as_uint(f[half * 8 + i].x);
        r[4 * i + 1] = __float_as_uint(f[half * 8 + i].y);
        r[4 * i + 2] = __float_as_uint(f[half * 8 + i].z);
        r[4 * i + 3] = __float_as_uint(f[half * 8 + i].w);
      }
      tmem_st32(tmem + lane_bits + TM_S + ch * 64 + half * 32, r);
    }
    tc_wait_st();
  }

  uint32_t mma_phase = 0, load_phase = 0;
  // thread 0 waits on `bar` (bounded); every thread learns the outcome (false: the CTA gives up)
  auto wait_bar = [&](uint64_t* bar, uint32_t parity, int where) -> bool {
    if (tid == 0) *ok_flag = mbar_wait(bar, parity, abort_flag, err, where) ? 1 : 0;
    __syncthreads();
    tc_fence_after();
    return *ok_flag != 0;
  };
  auto wait_mma = [&]() -> bool {
    const bool r = wait_bar(mma_bar, mma_phase, 40);
    mma_phase ^= 1;
    return r;
  };
  const uint32_t kq_a = smem_u32(kq), kd_a = smem_u32(kd), vb_a = smem_u32(vb), pt_a = smem_u32(pt),
                 rg_a = smem_u32(rg);
  bool ok = true;

  for (int c0 = 0; c0 < n && ok; c0 += C) {
    if (tid < C) {
      gc[tid] = g_next;
      bt[tid] = b_next;
    }
    // K and Q are in: MMA1 (the bounded wait on the TMA barriers, then every thread acquires them itself)
    if (!(ok = wait_bar(k_bar, load_phase, 41))) break;
    if (!(ok = wait_bar(qv_bar, load_phase, 42))) break;
    mbar_try_wait(k_bar, load_phase);
    mbar_try_wait(qv_bar, load_phase);
    load_phase ^= 1;
    // ---- MMA1: D1 = [K; Q] K^T
    if (warp == 1) {
      tc_fence_after();
      constexpr uint32_t id1 = idesc_bf16(128, 64);
      const bool issuer = elect_one();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t dsc = sw128_desc(kq_a + (kk >> 2) * 16384 + 32 * (kk & 3));
        if (issuer) tc_mma_bf16(tmem + TM_D1, dsc, dsc, id1, kk != 0);
      }
      if (issuer) tc_commit(mma_bar);
      __syncwarp();
    }
    // inclusive prefix sum of the 64 log-decays, then the per-token factors
    if (warp == 0) {
      float a = gc[lane], b = gc[lane + 32];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float ya = __shfl_up_sync(0xffffffffu, a, off), yb = __shfl_up_sync(0xffffffffu, b, off);
        if (lane >= off) { a += ya; b += yb; }
      }
      b += __shfl_sync(0xffffffffu, a, 31);
      gc[lane] = a;
      gc[lane + 32] = b;
      const float gl = __shfl_sync(0xffffffffu, b, 31);
      eg[lane] = expf(a);
      eg[lane + 32] = expf(b);
      ed[lane] = expf(gl - a);
      ed[lane + 32] = expf(gl - b);
    }
    __syncthreads();
    const float glast = gc[C - 1];
    // β V in place, e^{gc_last - gc} K into kd (MMA1 reads only K and Q): thread = (token, 16-byte piece)
    for (int i = tid; i < C * 16; i += THREADS) {
      const int t = i >> 4, c = i & 15, a = c >> 3;
      uint8_t* vp = swz(vb + a * 8192, t, c & 7);
      *reinterpret_cast<uint4*>(vp) = scale8(*reinterpret_cast<const uint4*>(vp), bt[t]);
      *reinterpret_cast<uint4*>(swz(kd + a * 8192, t, c & 7)) =
          scale8(*reinterpret_cast<const uint4*>(swz(kq + a * 16384, t, c & 7)), ed[t]);
    }
    if (tid == 0) tma_store_wait_read();   // the previous chunk's output tile has left the solve region
    if (!(ok = wait_mma())) break;
    // ---- D1 -> A (fp32, lanes 0-63) and P (bf16, lanes 64-127), columns 32 ch .. + 31
    {
      uint32_t r[32];
      tmem_ld32(tmem + lane_bits + TM_D1 + 32 * ch, r);
      tc_wait_ld();
      if (L < C) {
        const int i = L;
        const float gi = gc[i], bi = bt[i];
#pragma unroll
        for (int e4 = 0; e4 < 8; ++e4) {
          float4 w;
          float* wp = &w.x;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 32 * ch + 4 * e4 + e;
            wp[e] = i > j ? -bi * __uint_as_float(r[4 * e4 + e]) * exp_neg(fminf(gi - gc[j], 0.f)) : 0.f;
          }
          *reinterpret_cast<float4*>(&amat[i * PF + 32 * ch + 4 * e4]) = w;
        }
      } else {
        const int i = L - C;
        const float gi = gc[i];
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint32_t pk[4];
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const int j0 = 32 * ch + 8 * c8 + 2 * e2;
            pk[e2] = pack_bf2(
                i >= j0 ? __uint_as_float(r[8 * c8 + 2 * e2]) * exp_neg(fminf(gi - gc[j0], 0.f)) : 0.f,
                i >= j0 + 1 ? __uint_as_float(r[8 * c8 + 2 * e2 + 1]) * exp_neg(fminf(gi - gc[j0 + 1], 0.f)) : 0.f);
          }
          *reinterpret_cast<uint4*>(swz(pt, i, 4 * ch + c8)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    }
    __syncthreads();
    // ---- T = (I - A)^-1, diagonal 16 x 16 blocks (threads 0-63: block b, column j, by substitution) while the
    // other warps turn K into β e^gc K and Q into e^gc Q in place (MMA1, their last raw reader, is done)
    if (tid < 64) {
      const int b = tid >> 4, j = tid & 15;
      const int base = 16 * b;
      float col[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) col[i] = (i == j) ? 1.f : 0.f;
#pragma unroll
      for (int i = 1; i < 16; ++i) {
        if (i > j) {
          float acc = 0.f;
#pragma unroll
          for (int m = 0; m < 16; ++m)
            if (m < i) acc += amat[(base + i) * PF + base + m] * col[m];
          col[i] = acc;
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) tf[(base + i) * PF + base + j] = col[i];
    } else {
      for (int i = tid - 64; i < C * 16; i += THREADS - 64) {
        const int t = i >> 4, c = i & 15, a = c >> 3;
        uint8_t* kp = swz(kq + a * 16384, t, c & 7);
        uint8_t* qp = swz(kq + a * 16384 + 8192, t, c & 7);
        const float b0 = bt[t], e0 = eg[t];
        const uint4 x = *reinterpret_cast<const uint4*>(kp);
        uint4 y;   // β e^gc K, the product in the mma.sync form's order
        y.x = pack_bf2(bf_lo(x.x) * b0 * e0, bf_hi(x.x) * b0 * e0);
        y.y = pack_bf2(bf_lo(x.y) * b0 * e0, bf_hi(x.y) * b0 * e0);
        y.z = pack_bf2(bf_lo(x.z) * b0 * e0, bf_hi(x.z) * b0 * e0);
        y.w = pack_bf2(bf_lo(x.w) * b0 * e0, bf_hi(x.w) * b0 * e0);
        *reinterpret_cast<uint4*>(kp) = y;
        *reinterpret_cast<uint4*>(qp) = scale8(*reinterpret_cast<const uint4*>(qp), e0);
      }
      // T's blocks (0, 1) and (2, 3) above the diagonal are zero (the doubling steps multiply whole 32 x 32 blocks)
      for (int i = tid - 64; i < 2 * 16 * 16; i += THREADS - 64) {
        const int p = i >> 8, r = (i >> 4) & 15, c = i & 15;
        tf[(32 * p + r) * PF + 32 * p + 16 + c] = 0.f;
      }
    }
    __syncthreads();
    // doubling, step 1 (32 x 32 blocks p = 0, 1): X = T_{2p+1} A_{2p+1,2p} T_{2p}, via Z = A_{2p+1,2p} T_{2p}
    // staged in A's empty block (2p, 2p+1); thread = (p, row i, 2 columns)
    {
      const int p = tid >> 7, i = (tid >> 3) & 15, c2 = (tid & 7) * 2;
      const int r0 = 32 * p + 16, c0 = 32 * p;
      float z0 = 0.f, z1 = 0.f;
#pragma unroll
      for (int kx = 0; kx < 16; ++kx) {
        const float av = amat[(r0 + i) * PF + c0 + kx];
        const float2 tv = *reinterpret_cast<const float2*>(&tf[(c0 + kx) * PF + c0 + c2]);
        z0 += av * tv.x;
        z1 += av * tv.y;
      }
      *reinterpret_cast<float2*>(&amat[(c0 + i) * PF + r0 + c2]) = make_float2(z0, z1);
      __syncthreads();
      float x0 = 0.f, x1 = 0.f;
#pragma unroll
      for (int kx = 0; kx < 16; ++kx) {
        const float tv = tf[(r0 + i) * PF + r0 + kx];
        const float2 zv = *reinterpret_cast<const float2*>(&amat[(c0 + kx) * PF + r0 + c2]);
        x0 += tv * zv.x;
        x1 += tv * zv.y;
      }
      *reinterpret_cast<float2*>(&tf[(r0 + i) * PF + c0 + c2]) = make_float2(x0, x1);
    }
    __syncthreads();
    // doubling, step 2 (64 x 64): T_21 = T_22 A_21 T_11 with 32 x 32 blocks, via Z = A_21 T_11 staged in A's empty
    // upper-right block; thread = (row i, 4 columns)
    {
      const int i = tid >> 3, c4 = (tid & 7) * 4;
      float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int kx = 0; kx < 32; ++kx) {
        const float av = amat[(32 + i) * PF + kx];
        const float4 tv = *reinterpret_cast<const float4*>(&tf[kx * PF + c4]);
        z.x += av * tv.x;
        z.y += av * tv.y;
        z.z += av * tv.z;
        z.w += av * tv.w;
      }
      *reinterpret_cast<float4*>(&amat[i * PF + 32 + c4]) = z;
      __syncthreads();
      float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int kx = 0; kx < 32; ++kx) {
        const float tv = tf[(32 + i) * PF + 32 + kx];
        const float4 zv = *reinterpret_cast<const float4*>(&amat[kx * PF + 32 + c4]);
        y.x += tv * zv.x;
        y.y += tv * zv.y;
        y.z += tv * zv.z;
        y.w += tv * zv.w;
      }
      *reinterpret_cast<float4*>(&tf[(32 + i) * PF + c4]) = y;
    }
    __syncthreads();
    // T (bf16, zero above the diagonal) over A: 64 rows x 8 chunks, K-major
    for (int idx = tid; idx < C * 8; idx += THREADS) {
      const int i = idx >> 3, c = idx & 7;
      uint32_t pk[4];
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) {
        const int j = 8 * c + 2 * e2;
        pk[e2] = pack_bf2(j <= i ? tf[i * PF + j] : 0.f, j + 1 <= i ? tf[i * PF + j + 1] : 0.f);
      }
      *reinterpret_cast<uint4*>(swz(rg, i, c)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- MMA2: D1 = (β e^gc K)^T T^T = W^T, D2 = (β V)^T T^T = U^T
    if (warp == 1) {
      tc_fence_after();
      constexpr uint32_t id2 = idesc_bf16(128, 64) | A_MN;
      const bool issuer = elect_one();
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        const uint64_t bd = sw128_desc(rg_a + 32 * kk);
        const uint64_t a1 = mn_desc(kq_a + kk * 2048, 16384), a2 = mn_desc(vb_a + kk * 2048, 8192);
        if (issuer) {
          tc_mma_bf16(tmem + TM_D1, a1, bd, id2, kk != 0);
          tc_mma_bf16(tmem + TM_D2, a2, bd, id2, kk != 0);
        }
      }
      if (issuer) tc_commit(mma_bar);
      __syncwarp();
    }
    if (!(ok = wait_mma())) break;
    const bool more = c0 + C < n;
    if (loader && more) load_k(c0 + C);   // the K slots (β e^gc K) were last read by MMA2
    // ---- -W^T (bf16) over β V: key row L, tokens 32 ch .. + 31; S (bf16) over T: value atom ch, key row L; the
    // state in tensor memory scaled by e^{gc_last} for MMA5
    {
      uint32_t r[32];
      tmem_ld32(tmem + lane_bits + TM_D1 + 32 * ch, r);
      tc_wait_ld();
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint4 y;
        y.x = pack_bf2(-__uint_as_float(r[8 * c8 + 0]), -__uint_as_float(r[8 * c8 + 1]));
        y.y = pack_bf2(-__uint_as_float(r[8 * c8 + 2]), -__uint_as_float(r[8 * c8 + 3]));
        y.z = pack_bf2(-__uint_as_float(r[8 * c8 + 4]), -__uint_as_float(r[8 * c8 + 5]));
        y.w = pack_bf2(-__uint_as_float(r[8 * c8 + 6]), -__uint_as_float(r[8 * c8 + 7]));
        *reinterpret_cast<uint4*>(swz(vb, L, 4 * ch + c8)) = y;
      }
      const float el = expf(glast);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint32_t ta = tmem + lane_bits + TM_S + 64 * ch + 32 * half;
        tmem_ld32(ta, r);
        tc_wait_ld();
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint4 y;
          y.x = pack_bf2(__uint_as_float(r[8 * c8 + 0]), __uint_as_float(r[8 * c8 + 1]));
          y.y = pack_bf2(__uint_as_float(r[8 * c8 + 2]), __uint_as_float(r[8 * c8 + 3]));
          y.z = pack_bf2(__uint_as_float(r[8 * c8 + 4]), __uint_as_float(r[8 * c8 + 5]));
          y.w = pack_bf2(__uint_as_float(r[8 * c8 + 6]), __uint_as_float(r[8 * c8 + 7]));
          *reinterpret_cast<uint4*>(swz(rg + ch * 16384, L, 4 * half + c8)) = y;
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * el);
        tmem_st32(ta, r);
      }
      tc_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- MMA3: D2 += S^T (-W^T) = V'^T
    if (warp == 1) {
      tc_fence_after();
      constexpr uint32_t id3 = idesc_bf16(128, 64) | A_MN | B_MN;
      const bool issuer = elect_one();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t a = mn_desc(rg_a + kk * 2048, 16384), b = mn_desc(vb_a + kk * 2048, 8192);
        if (issuer) tc_mma_bf16(tmem + TM_D2, a, b, id3, 1);
      }
      if (issuer) tc_commit(mma_bar);
      __syncwarp();
    }
    if (!(ok = wait_mma())) break;
    // ---- V'^T (bf16) over -W^T: value row L, tokens 32 ch .. + 31 (K-major: the A of O^T, the B of the update)
    {
      uint32_t r[32];
      tmem_ld32(tmem + lane_bits + TM_D2 + 32 * ch, r);
      tc_wait_ld();
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint4 y;
        y.x = pack_bf2(__uint_as_float(r[8 * c8 + 0]), __uint_as_float(r[8 * c8 + 1]));
        y.y = pack_bf2(__uint_as_float(r[8 * c8 + 2]), __uint_as_float(r[8 * c8 + 3]));
        y.z = pack_bf2(__uint_as_float(r[8 * c8 + 4]), __uint_as_float(r[8 * c8 + 5]));
        y.w = pack_bf2(__uint_as_float(r[8 * c8 + 6]), __uint_as_float(r[8 * c8 + 7]));
        *reinterpret_cast<uint4*>(swz(vb, L, 4 * ch + c8)) = y;
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- MMA4: D1 = S^T (e^gc Q)^T + V'^T P^T = O^T;  MMA5: S += (e^{gc_last - gc} K)^T V'
    if (warp == 1) {
      tc_fence_after();
      constexpr uint32_t id4 = idesc_bf16(128, 64) | A_MN;
      constexpr uint32_t id4b = idesc_bf16(128, 64);
      constexpr uint32_t id5 = idesc_bf16(128, 128) | A_MN;
      const bool issuer = elect_one();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t a = mn_desc(rg_a + kk * 2048, 16384),
                       b = sw128_desc(kq_a + 8192 + (kk >> 2) * 16384 + 32 * (kk & 3));
        if (issuer) tc_mma_bf16(tmem + TM_D1, a, b, id4, kk != 0);
      }
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        const uint64_t a = sw128_desc(vb_a + 32 * kk), b = sw128_desc(pt_a + 32 * kk);
        if (issuer) tc_mma_bf16(tmem + TM_D1, a, b, id4b, 1);
      }
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        const uint64_t a = mn_desc(kd_a + kk * 2048, 8192), b = sw128_desc(vb_a + 32 * kk);
        if (issuer) tc_mma_bf16(tmem + TM_S, a, b, id5, 1);
      }
      if (issuer) tc_commit(mma_bar);
      __syncwarp();
    }
    if (tid < C) {   // the next chunk's gates
      const bool valid = c0 + C + tid < n;
      g_next = valid ? g[(rbase + c0 + C + tid) * NH + h] : 0.f;
      b_next = valid ? __bfloat162float(beta[(rbase + c0 + C + tid) * NH + h]) : 0.f;
    }
    if (!(ok = wait_mma())) break;
    if (loader && more) load_qv(c0 + C);   // the Q and V slots are free now
    // ---- O^T -> bf16 (scaled; zeros past stop) -> the output tile over S bf16, laid out as the loads -> TMA store
    {
      uint32_t r[32];
      tmem_ld32(tmem + lane_bits + TM_D1 + 32 * ch, r);
      tc_wait_ld();
      __nv_bfloat16* ot = reinterpret_cast<__nv_bfloat16*>(rg + (L >> 6) * 8192);
      const int cl = L & 63;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int t = 32 * ch + e;
        const float val = c0 + t < stop ? __uint_as_float(r[e]) * scale : 0.f;
        ot[(sw128_offset(t, cl >> 3) >> 1) + (cl & 7)] = f2bf(val);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (loader) {
      tma_store_4d(&tm_o, rg, 0, h, c0, row);
      tma_store_4d(&tm_o, rg + 8192, 64, h, c0, row);
      tma_store_commit();
    }
  }
  if (loader) {
    tma_store_wait_all();
    // a CTA that gave up waits (bounded) for the loads it issued before its shared memory goes away: load i of a
    // barrier completes its phase i, and each load was issued after the previous one of its barrier had landed, so
    // waiting for the last one suffices
    const uint64_t t0 = global_ns();
    while (k_issued && !mbar_try_wait(k_bar, (k_issued - 1) & 1) && global_ns() - t0 < kWaitNs) {
    }
    while (qv_issued && !mbar_try_wait(qv_bar, (qv_issued - 1) & 1) && global_ns() - t0 < kWaitNs) {
    }
  }

  if (ok && out_tables) {
    const int opage = out_tables[(size_t)row * out_table_stride + flat / heads_per_page];
    float* s_out = reinterpret_cast<float*>(pool + (int64_t)opage * page_bytes + (flat % heads_per_page) * STATE_BYTES);
    float4* dst = reinterpret_cast<float4*>(s_out + (size_t)L * D + ch * 64);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t r[32];
      tmem_ld32(tmem + lane_bits + TM_S + 64 * ch + 32 * half, r);
      tc_wait_ld();
#pragma unroll
      for (int i = 0; i < 8; ++i)
        dst[half * 8 + i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                        __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// q, k, v or o (b, n, 16, 128) bf16 as a 4-D tensor map (channel, head, token, row); boxes of 64 channels x 1 head x
// 64 tokens, 128-byte swizzle: one box is one 64-column atom of a chunk's tile
int tile_map(CUtensorMap* map, const void* base, int b, int n) {
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)NH, (uint64_t)n, (uint64_t)b};
  const uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)NH * D * 2, (uint64_t)n * NH * D * 2};
  const uint32_t box[4] = {64, 1, (uint32_t)C, 1};
  return make_tmap_nd(map, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace gdnt
}  // namespace jb

extern "C" int jb_gdn_scan_tc(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                              const uint16_t* beta, uint16_t* o, int b, int n, void* pool, int64_t page_bytes,
                              const int32_t* tables, int table_stride, int first_head, int heads_per_page,
                              const int32_t* last, const int32_t* out_tables, int out_table_stride, void* stream) {
  using namespace jb;
  JB_REQUIRE(q && k && v && g && beta && o && pool && tables, "jb_gdn_scan_tc: null pointer");
  JB_REQUIRE(b > 0 && n > 0, "jb_gdn_scan_tc: b %d, n %d", b, n);
  JB_REQUIRE(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
               reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(pool)) & 15) == 0,
             "jb_gdn_scan_tc: q, k, v, o and the pool must be 16-byte aligned");
  JB_REQUIRE(page_bytes % 16 == 0, "jb_gdn_scan_tc: page size %lld is not a multiple of 16", (long long)page_bytes);
  JB_REQUIRE(heads_per_page > 0 && (int64_t)heads_per_page * (int64_t)gdnc::STATE_BYTES <= page_bytes,
             "jb_gdn_scan_tc: %d heads per page do not fit pages of %lld bytes", heads_per_page,
             (long long)page_bytes);
  JB_REQUIRE(first_head >= 0 && (first_head + gdnc::NH - 1) / heads_per_page < table_stride,
             "jb_gdn_scan_tc: heads %d.. reach past the block table (%d entries)", first_head, table_stride);
  CUtensorMap tq, tk, tv, to;
  int st = gdnt::tile_map(&tq, q, b, n);
  if (!st) st = gdnt::tile_map(&tk, k, b, n);
  if (!st) st = gdnt::tile_map(&tv, v, b, n);
  if (!st) st = gdnt::tile_map(&to, o, b, n);
  if (st) return st;
  st = gdnc::configure(gdnt::scan_kernel, gdnt::ALLOC, "gdn scan_kernel (tcgen05)");
  if (st) return st;
  launch_pdl(gdnt::scan_kernel, b * gdnc::NH, gdnt::THREADS, gdnt::ALLOC, (cudaStream_t)stream,
      tq, tk, tv, to, g, reinterpret_cast<const __nv_bfloat16*>(beta), n, static_cast<uint8_t*>(pool), page_bytes,
      tables, table_stride, first_head, heads_per_page, last, out_tables, out_table_stride, device_status_word());
  return check_launch("gdn scan_kernel (tcgen05)");
}
