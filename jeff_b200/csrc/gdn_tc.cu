// S2 on tcgen05: the gated delta rule over 64-token chunks with every chunk product on the 5th-generation tensor
// cores, the fp32 state resident in tensor memory, each (row, head) resuming from its state in the prefix pool (the
// chunked form of fla's chunk_gated_delta_rule, which the reference's batched path calls at batched_path.py:282-288,
// :322-324, and of transformers' torch_chunk_gated_delta_rule on its standard path).
//
// Per chunk of C = 64 tokens (gc = cumulative log-decay within the chunk, Γ_ij = exp(gc_i - gc_j)), the same
// quantities and bf16 rounding points as the mma.sync form in gdn_chunk.cu:
//   A = strictly lower part of -diag(β) K K^T ∘ Γ, T = (I - A)^-1 (fp32, 16 x 16 blocked substitution)
//   W = T (β e^gc K), U = T (β V), V' = U - W S, O = scale ((e^gc Q) S + (Q K^T ∘ Γ, causal) V'),
//   S <- e^{gc_last} S + (e^{gc_last - gc} K)^T V'.
// Tensor memory (256 columns; 128 lanes): S (key lanes x 128 value columns, fp32) in columns 0-127, D1 in 128-191,
// D2 in 192-255. The products are issued by one thread as M = 128 tcgen05 MMAs, transposed where that puts 128 rows
// on the lanes:
//   MMA1  D1 = [K; Q] K^T            (lanes 0-63: K K^T rows, 64-127: Q K^T rows; the stacked A is K and Q tiles
//                                     laid out back to back)
//   MMA2  D1 = (β e^gc K)^T T^T = W^T,  D2 = (β V)^T T^T = U^T
//   MMA3  D2 += S^T (-W^T)          -> V'^T
//   MMA4  D1 = S^T (e^gc Q)^T + V'^T P^T = O^T
//   MMA5  S += (e^{gc_last - gc} K)^T V'   (S scaled by e^{gc_last} in tensor memory beforehand)
// The eight warps read each result out of tensor memory (warp w: lanes 32 (w % 4) .., columns half w / 4) and write
// the next operands into shared memory in the 128-byte swizzled layouts the MMAs read (K-major or MN-major). The T
// solve runs on the CUDA cores. Every tile is 64 tokens x 128 elements as two 64-column swizzle atoms; one CTA of
// 8 warps per (row, head) with about 108 KB of shared memory, so two CTAs share an SM and one's solve overlaps the
// other's products. The single-thread waits on MMA completion are bounded (%globaltimer, 2 s): on expiry the CTA
// records JB_DEV_TIMEOUT | 40 in the device status word and returns.

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
                                   // the output staging (64 tokens x 128 values, pitch 136)
constexpr int R_BYTES = 2 * C * PF * 4;
constexpr int OFF_G = OFF_R + R_BYTES;   // gc, e^gc, e^{gc_last - gc}, β (64 floats each)
constexpr int OFF_MISC = OFF_G + 4 * C * 4;
constexpr int BYTES = OFF_MISC + 64;
constexpr int ALLOC = BYTES + 1024;
constexpr int OPITCH = 136;              // output staging pitch (bf16 elements)
static_assert(2 * D * 128 <= R_BYTES, "S bf16 fits the solve region");
static_assert(C * OPITCH * 2 <= R_BYTES, "output staging fits the solve region");
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

// 16-byte chunk c (0..7) of row r of a 128-byte-row swizzled tile
__device__ __forceinline__ uint8_t* swz(uint8_t* tile, int r, int c) { return tile + sw128_offset(r, c); }

__global__ void __launch_bounds__(THREADS, 2)
    scan_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
                const __nv_bfloat16* __restrict__ beta, __nv_bfloat16* __restrict__ o, int n,
                uint8_t* __restrict__ pool, int64_t page_bytes, const int* __restrict__ tables, int table_stride,
                int first_head, int heads_per_page, const int* __restrict__ last, const int* __restrict__ out_tables,
                int out_table_stride, int* err) {
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_MISC + 8);
  volatile int* ok_flag = reinterpret_cast<volatile int*>(sm + OFF_MISC + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + OFF_MISC + 16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, ch = warp >> 2;
  const int L = 32 * qd + lane;                  // this thread's tensor-memory lane
  const uint32_t lane_bits = (uint32_t)(32 * qd) << 16;
  const int row = blockIdx.x / NH, h = blockIdx.x % NH;
  const int flat = first_head + h;
  const float scale = rsqrtf((float)D);
  const int stop = last ? min(last[row] + 1, n) : n;   // outputs past stop are written as zeros
  const size_t rbase = (size_t)row * n;

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }

  // raw tiles of the chunk at c0 (zero past its end): which bit 0 K, bit 1 Q, bit 2 V
  auto issue_loads = [&](int c0, int which) {
    const int len = min(C, n - c0);
    for (int i = tid; i < 3 * C * 16; i += THREADS) {
      const int part = i / (C * 16), rem = i % (C * 16);
      if (!((which >> part) & 1)) continue;
      const int t = rem >> 4, c = rem & 15, a = c >> 3;
      const bool valid = t < len;
      const __nv_bfloat16* src = (part == 0 ? k : part == 1 ? q : v) +
                                 ((rbase + c0 + (valid ? t : 0)) * NH + h) * D + c * 8;
      uint8_t* tile = part == 0 ? kq + a * 16384 : part == 1 ? kq + a * 16384 + 8192 : vb + a * 8192;
      gdnc::cp_async16(swz(tile, t, c & 7), src, valid);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue_loads(0, 7);
  // gates of the next chunk, held in registers until it starts
  float g_next = 0.f, b_next = 0.f;
  if (tid < C) {
    const bool valid = tid < n;
    g_next = valid ? g[(rbase + tid) * NH + h] : 0.f;
    b_next = valid ? __bfloat162float(beta[(rbase + tid) * NH + h]) : 0.f;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // the state of this (row, head) from its pool page into tensor memory: lane = key row, columns = value
  {
    const int page = tables[(size_t)row * table_stride + flat / heads_per_page];
    const float* s_in =
        reinterpret_cast<const float*>(pool + (int64_t)page * page_bytes + (flat % heads_per_page) * STATE_BYTES);
    const float4* src = reinterpret_cast<const float4*>(s_in + (size_t)L * D + ch * 64);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 f = src[half * 8 + i];
        r[4 * i] = __float_as_uint(f.x);
        r[4 * i + 1] = __float_as_uint(f.y);
        r[4 * i + 2] = __float_as_uint(f.z);
        r[4 * i + 3] = __float_as_uint(f.w);
      }
      tmem_st32(tmem + lane_bits + TM_S + ch * 64 + half * 32, r);
    }
    tc_wait_st();
  }

  uint32_t phase = 0;
  // one thread waits for the MMAs committed last; every thread learns the outcome (false: the CTA gives up)
  auto wait_mma = [&]() -> bool {
    if (tid == 0) *ok_flag = mbar_wait(mma_bar, phase, abort_flag, err, 40) ? 1 : 0;
    phase ^= 1;
    __syncthreads();
    tc_fence_after();
    return *ok_flag != 0;
  };
  const uint32_t kq_a = smem_u32(kq), kd_a = smem_u32(kd), vb_a = smem_u32(vb), pt_a = smem_u32(pt),
                 rg_a = smem_u32(rg);
  bool ok = true;

  for (int c0 = 0; c0 < n && ok; c0 += C) {
    const int len = min(C, n - c0);
    if (tid < C) {
      gc[tid] = g_next;
      bt[tid] = b_next;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- MMA1: D1 = [K; Q] K^T
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t id1 = idesc_bf16(128, 64);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t a = kq_a + (kk >> 2) * 16384 + 32 * (kk & 3);
        tc_mma_bf16(tmem + TM_D1, sw128_desc(a), sw128_desc(a), id1, kk != 0);
      }
      tc_commit(mma_bar);
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
    }
    __syncthreads();
    const float glast = gc[C - 1];
    if (tid < C) {
      eg[tid] = expf(gc[tid]);
      ed[tid] = expf(glast - gc[tid]);
    }
    __syncthreads();
    // β V in place, e^{gc_last - gc} K into kd (MMA1 reads only K and Q)
    for (int i = tid; i < 2 * C * 16; i += THREADS) {
      const int part = i / (C * 16), rem = i % (C * 16);
      const int t = rem >> 4, c = rem & 15, a = c >> 3;
      uint8_t* src = part == 0 ? swz(vb + a * 8192, t, c & 7) : swz(kq + a * 16384, t, c & 7);
      uint8_t* dst = part == 0 ? src : swz(kd + a * 8192, t, c & 7);
      const float f = part == 0 ? bt[t] : ed[t];
      const uint4 x = *reinterpret_cast<const uint4*>(src);
      uint4 y;
      y.x = pack_bf2(bf_lo(x.x) * f, bf_hi(x.x) * f);
      y.y = pack_bf2(bf_lo(x.y) * f, bf_hi(x.y) * f);
      y.z = pack_bf2(bf_lo(x.z) * f, bf_hi(x.z) * f);
      y.w = pack_bf2(bf_lo(x.w) * f, bf_hi(x.w) * f);
      *reinterpret_cast<uint4*>(dst) = y;
    }
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
            const float decay = expf(fminf(gi - gc[j], 0.f));
            wp[e] = i > j ? -bi * __uint_as_float(r[4 * e4 + e]) * decay : 0.f;
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
            const float d0 = expf(fminf(gi - gc[j0], 0.f)), d1 = expf(fminf(gi - gc[j0 + 1], 0.f));
            pk[e2] = pack_bf2(i >= j0 ? __uint_as_float(r[8 * c8 + 2 * e2]) * d0 : 0.f,
                              i >= j0 + 1 ? __uint_as_float(r[8 * c8 + 2 * e2 + 1]) * d1 : 0.f);
          }
          *reinterpret_cast<uint4*>(swz(pt, i, 4 * ch + c8)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    }
    __syncthreads();
    // ---- T = (I - A)^-1: diagonal 16 x 16 blocks (threads 0-63: block b, column j) while the other warps turn K
    // into β e^gc K and Q into e^gc Q in place (MMA1, their last raw reader, is done)
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
      for (int i = tid - 64; i < 2 * C * 16; i += THREADS - 64) {
        const int part = i / (C * 16), rem = i % (C * 16);
        const int t = rem >> 4, c = rem & 15, a = c >> 3;
        uint8_t* p = swz(kq + a * 16384 + part * 8192, t, c & 7);
        const uint4 x = *reinterpret_cast<const uint4*>(p);
        uint4 y;
        if (part == 0) {   // β e^gc K, the product in the mma.sync form's order
          const float b0 = bt[t], e0 = eg[t];
          y.x = pack_bf2(bf_lo(x.x) * b0 * e0, bf_hi(x.x) * b0 * e0);
          y.y = pack_bf2(bf_lo(x.y) * b0 * e0, bf_hi(x.y) * b0 * e0);
          y.z = pack_bf2(bf_lo(x.z) * b0 * e0, bf_hi(x.z) * b0 * e0);
          y.w = pack_bf2(bf_lo(x.w) * b0 * e0, bf_hi(x.w) * b0 * e0);
        } else {
          const float e0 = eg[t];
          y.x = pack_bf2(bf_lo(x.x) * e0, bf_hi(x.x) * e0);
          y.y = pack_bf2(bf_lo(x.y) * e0, bf_hi(x.y) * e0);
          y.z = pack_bf2(bf_lo(x.z) * e0, bf_hi(x.z) * e0);
          y.w = pack_bf2(bf_lo(x.w) * e0, bf_hi(x.w) * e0);
        }
        *reinterpret_cast<uint4*>(p) = y;
      }
    }
    __syncthreads();
    // off-diagonal blocks by distance from the diagonal (each distance one parallel step): thread = (block column c,
    // row i, 4 adjacent columns); T_rc = T_rr (sum_{m=c}^{r-1} A_rm T_mc), the inner sum staged in A's empty upper
    // part
    {
      const int bc = tid >> 6, i = (tid >> 2) & 15, q4 = (tid & 3) * 4;
      for (int d = 1; d < 4; ++d) {
        const int c = bc, r = c + d;
        const bool active = r < 4;
        if (active) {
          float4 tmp = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int m = c; m < r; ++m)
#pragma unroll
            for (int kx = 0; kx < 16; ++kx) {
              const float av = amat[(16 * r + i) * PF + 16 * m + kx];
              const float4 tv = *reinterpret_cast<const float4*>(&tf[(16 * m + kx) * PF + 16 * c + q4]);
              tmp.x += av * tv.x;
              tmp.y += av * tv.y;
              tmp.z += av * tv.z;
              tmp.w += av * tv.w;
            }
          *reinterpret_cast<float4*>(&amat[(16 * c + i) * PF + 16 * r + q4]) = tmp;
        }
        __syncthreads();
        if (active) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int kx = 0; kx < 16; ++kx) {
            const float tv = tf[(16 * r + i) * PF + 16 * r + kx];
            const float4 av = *reinterpret_cast<const float4*>(&amat[(16 * c + kx) * PF + 16 * r + q4]);
            acc.x += tv * av.x;
            acc.y += tv * av.y;
            acc.z += tv * av.z;
            acc.w += tv * av.w;
          }
          *reinterpret_cast<float4*>(&tf[(16 * r + i) * PF + 16 * c + q4]) = acc;
        }
        __syncthreads();
      }
    }
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
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t id2 = idesc_bf16(128, 64) | A_MN;
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        const uint64_t bd = sw128_desc(rg_a + 32 * kk);
        tc_mma_bf16(tmem + TM_D1, mn_desc(kq_a + kk * 2048, 16384), bd, id2, kk != 0);
        tc_mma_bf16(tmem + TM_D2, mn_desc(vb_a + kk * 2048, 8192), bd, id2, kk != 0);
      }
      tc_commit(mma_bar);
    }
    if (!(ok = wait_mma())) break;
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
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t id3 = idesc_bf16(128, 64) | A_MN | B_MN;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        tc_mma_bf16(tmem + TM_D2, mn_desc(rg_a + kk * 2048, 16384), mn_desc(vb_a + kk * 2048, 8192), id3, 1);
      tc_commit(mma_bar);
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
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t id4 = idesc_bf16(128, 64) | A_MN;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        tc_mma_bf16(tmem + TM_D1, mn_desc(rg_a + kk * 2048, 16384),
                    sw128_desc(kq_a + 8192 + (kk >> 2) * 16384 + 32 * (kk & 3)), id4, kk != 0);
      constexpr uint32_t id4b = idesc_bf16(128, 64);
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk)
        tc_mma_bf16(tmem + TM_D1, sw128_desc(vb_a + 32 * kk), sw128_desc(pt_a + 32 * kk), id4b, 1);
      constexpr uint32_t id5 = idesc_bf16(128, 128) | A_MN;
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk)
        tc_mma_bf16(tmem + TM_S, mn_desc(kd_a + kk * 2048, 8192), sw128_desc(vb_a + 32 * kk), id5, 1);
      tc_commit(mma_bar);
    }
    // the next chunk's K tile loads into the K slots (β e^gc K was last read by MMA2)
    const bool more = c0 + C < n;
    if (more) issue_loads(c0 + C, 1);
    if (tid < C) {
      const bool valid = c0 + C + tid < n;
      g_next = valid ? g[(rbase + c0 + C + tid) * NH + h] : 0.f;
      b_next = valid ? __bfloat162float(beta[(rbase + c0 + C + tid) * NH + h]) : 0.f;
    }
    if (!(ok = wait_mma())) break;
    if (more) issue_loads(c0 + C, 6);   // Q and V slots are free now
    // ---- O^T -> bf16 (scaled) -> staging [token][value] over S bf16 -> 16-byte stores of each token's 128 values
    __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(rg);
    {
      uint32_t r[32];
      tmem_ld32(tmem + lane_bits + TM_D1 + 32 * ch, r);
      tc_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) stg[(32 * ch + e) * OPITCH + L] = f2bf(__uint_as_float(r[e]) * scale);
    }
    tc_fence_before();
    __syncthreads();
    for (int idx = tid; idx < C * 16; idx += THREADS) {
      const int t = idx >> 4, c = idx & 15;
      if (t < len) {
        const size_t tok = rbase + c0 + t;
        const uint4 val = c0 + t < stop ? *reinterpret_cast<const uint4*>(&stg[t * OPITCH + 8 * c])
                                        : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(o + (tok * NH + h) * D + 8 * c) = val;
      }
    }
    __syncthreads();
  }
  asm volatile("cp.async.wait_all;" ::: "memory");

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
  int st = gdnc::configure(gdnt::scan_kernel, gdnt::ALLOC, "gdn scan_kernel (tcgen05)");
  if (st) return st;
  gdnt::scan_kernel<<<b * gdnc::NH, gdnt::THREADS, gdnt::ALLOC, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
      reinterpret_cast<const __nv_bfloat16*>(v), g, reinterpret_cast<const __nv_bfloat16*>(beta),
      reinterpret_cast<__nv_bfloat16*>(o), n, static_cast<uint8_t*>(pool), page_bytes, tables, table_stride,
      first_head, heads_per_page, last, out_tables, out_table_stride, device_status_word());
  return check_launch("gdn scan_kernel (tcgen05)");
}
