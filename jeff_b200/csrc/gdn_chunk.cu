// S2 (chunked): the gated delta rule over 64-token chunks on tensor cores, each (row, head) resuming from its state
// in the prefix pool (the chunked form of the reference's standard path, transformers torch_chunk_gated_delta_rule,
// and of fla's chunk_gated_delta_rule that the reference's batched path calls, batched_path.py:282-288, :322-324).
//
// Per chunk of C = 64 tokens (gc = cumulative log-decay within the chunk, Γ_ij = exp(gc_i - gc_j)):
//   A   = strictly lower part of -diag(β) K K^T ∘ Γ            T = (I - A)^-1  (16 x 16 blocked substitution, fp32)
//   U   = T (diag(β) V)        W = T (diag(β e^gc) K)           V' = U - W S
//   O   = scale ((diag(e^gc) Q) S + (Q K^T ∘ Γ, causal incl. diagonal) V')
//   S  <- e^{gc_last} S + (diag(e^{gc_last - gc}) K)^T V'
// One CTA (8 warps) per (row, head). The fp32 state S (128 key x 128 value) lives in registers as mma accumulators
// (warp w: key rows 16w .. 16w + 15), with a bf16 copy in shared memory as the operand of the next chunk; every
// product is a bf16 mma.sync with fp32 accumulation (the operand roundings of fla's chunk kernel). Padding tokens of a
// partial chunk are zero (K = Q = V = 0, g = β = 0), which leaves S unchanged.

namespace jb {
namespace gdnc {

constexpr int C = 64, D = 128, NH = 16;
constexpr int P16 = D + 8;              // bf16 row pitch (elements) of 128-wide tiles: 272 B, ldmatrix conflict-free
constexpr int P64 = C + 8;              // bf16 row pitch of 64-wide tiles: 144 B
constexpr int PF = C + 4;               // fp32 row pitch of 64-wide tiles (rows 16-byte aligned)
constexpr size_t STATE_BYTES = (size_t)D * D * 4;

struct Smem {
  __nv_bfloat16 ks[C * P16];    // K, then W
  __nv_bfloat16 qs[C * P16];    // Q, then e^gc Q
  __nv_bfloat16 vs[C * P16];    // V, then β V
  __nv_bfloat16 kb[C * P16];    // β e^gc K, then V'
  __nv_bfloat16 kd[C * P16];    // e^{gc_last - gc} K
  __nv_bfloat16 sb[D * P16];    // bf16 copy of S (key rows)
  float amat[C * PF];           // A (fp32)
  float tf[C * PF];             // T (fp32)
  __nv_bfloat16 ts[C * P64];    // T (bf16)
  __nv_bfloat16 ps[C * P64];    // Q K^T ∘ Γ, causal (bf16)
  float gc[C];
  float eg[C];                  // e^gc per token
  float ed[C];                  // e^{gc_last - gc} per token
  float beta[C];
};

__device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm4(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm4t(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// A fragment (16 x 16) at (r0, c0) of a row-major bf16 matrix (pitch in elements)
__device__ __forceinline__ void frag_a(const __nv_bfloat16* m, int pitch, int r0, int c0, uint32_t (&a)[4]) {
  const int l = threadIdx.x & 31;
  ldsm4(m + (size_t)(r0 + (l & 15)) * pitch + c0 + (l >> 4) * 8, a);
}
// A fragment (16 m x 16 k) of the transpose of a row-major [k][m] matrix
__device__ __forceinline__ void frag_a_t(const __nv_bfloat16* m, int pitch, int m0, int k0, uint32_t (&a)[4]) {
  const int l = threadIdx.x & 31, i = l >> 3;
  ldsm4t(m + (size_t)(k0 + (i >> 1) * 8 + (l & 7)) * pitch + m0 + (i & 1) * 8, a);
}
// B fragments of two n-blocks (n0, n0 + 8) x k16 from a row-major [n][k] matrix: b[0], b[1] for n0; b[2], b[3] n0+8
__device__ __forceinline__ void frag_b_nk(const __nv_bfloat16* m, int pitch, int n0, int k0, uint32_t (&b)[4]) {
  const int l = threadIdx.x & 31, i = l >> 3;
  ldsm4(m + (size_t)(n0 + (i >> 1) * 8 + (l & 7)) * pitch + k0 + (i & 1) * 8, b);
}
// B fragments of two n-blocks x k16 from a row-major [k][n] matrix
__device__ __forceinline__ void frag_b_kn(const __nv_bfloat16* m, int pitch, int n0, int k0, uint32_t (&b)[4]) {
  const int l = threadIdx.x & 31, i = l >> 3;
  ldsm4t(m + (size_t)(k0 + (i & 1) * 8 + (l & 7)) * pitch + n0 + (i >> 1) * 8, b);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}

__global__ void __launch_bounds__(256, 1) chunk_kernel(const __nv_bfloat16* __restrict__ q,
                                                       const __nv_bfloat16* __restrict__ k,
                                                       const __nv_bfloat16* __restrict__ v,
                                                       const float* __restrict__ g,
                                                       const __nv_bfloat16* __restrict__ beta,
                                                       __nv_bfloat16* __restrict__ o, int n, uint8_t* __restrict__ pool,
                                                       int64_t page_bytes, const int* __restrict__ tables,
                                                       int table_stride, int first_head, int heads_per_page,
                                                       const int* __restrict__ last,
                                                       const int* __restrict__ out_tables, int out_table_stride) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int row = blockIdx.x / NH, h = blockIdx.x % NH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gr = lane >> 2, tq = lane & 3;
  const int flat = first_head + h;
  const float scale = rsqrtf((float)D);
  const int stop = last ? min(last[row] + 1, n) : n;   // outputs past stop are written as zeros

  // K, Q, V tiles of the chunk at c0 (zero past its end) into ks / qs / vs, asynchronously
  auto issue_loads = [&](int c0) {
    const int len = min(C, n - c0);
    for (int i = threadIdx.x; i < 3 * C * (D / 8); i += 256) {
      const int which = i / (C * (D / 8));
      const int rem = i % (C * (D / 8));
      const int t = rem / (D / 8), ch = rem % (D / 8);
      const bool valid = t < len;
      const size_t tok = (size_t)row * n + c0 + (valid ? t : 0);
      const __nv_bfloat16* src = (which == 0 ? k : which == 1 ? q : v) + (tok * NH + h) * D + ch * 8;
      __nv_bfloat16* dst = (which == 0 ? sm.ks : which == 1 ? sm.qs : sm.vs) + t * P16 + ch * 8;
      cp_async16(dst, src, valid);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue_loads(0);   // in flight while the state loads

  // ---- the initial state: fp32 accumulators (warp w: key rows 16w + gr (+8), value cols 8nb + 2tq (+1))
  float s[16][4];
  {
    const int page = tables[(size_t)row * table_stride + flat / heads_per_page];
    const float* s_in = reinterpret_cast<const float*>(pool + (int64_t)page * page_bytes +
                                                       (flat % heads_per_page) * STATE_BYTES);
    const int r0 = 16 * warp + gr;
#pragma unroll
    for (int nb = 0; nb < 16; ++nb) {
      const float2 lo = *reinterpret_cast<const float2*>(s_in + (size_t)r0 * D + nb * 8 + 2 * tq);
      const float2 hi = *reinterpret_cast<const float2*>(s_in + (size_t)(r0 + 8) * D + nb * 8 + 2 * tq);
      s[nb][0] = lo.x; s[nb][1] = lo.y; s[nb][2] = hi.x; s[nb][3] = hi.y;
    }
  }

  const int wr = warp & 3;          // 16-row block of the 64-row tiles this warp computes
  const int wc = warp >> 2;         // column half (64 of 128) of the 64 x 128 tiles

  for (int c0 = 0; c0 < n; c0 += C) {
    const int len = min(C, n - c0);
    // ---- S (bf16) for this chunk's operands; K, Q, V tiles (zero past len)
#pragma unroll
    for (int nb = 0; nb < 16; ++nb) {
      const int r0 = 16 * warp + gr, cc = nb * 8 + 2 * tq;
      *reinterpret_cast<uint32_t*>(&sm.sb[r0 * P16 + cc]) = pack_bf2(s[nb][0], s[nb][1]);
      *reinterpret_cast<uint32_t*>(&sm.sb[(r0 + 8) * P16 + cc]) = pack_bf2(s[nb][2], s[nb][3]);
    }
    // (this chunk's K, Q, V were issued before the state load or during the previous chunk's state update)
    if (threadIdx.x < C) {
      const int t = threadIdx.x;
      const size_t tok = (size_t)row * n + c0 + t;
      sm.gc[t] = t < len ? g[tok * NH + h] : 0.f;
      sm.beta[t] = t < len ? __bfloat162float(beta[tok * NH + h]) : 0.f;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (warp == 0) {   // inclusive prefix sum of the 64 log-decays
      float a = sm.gc[lane], b = sm.gc[lane + 32];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float ya = __shfl_up_sync(0xffffffffu, a, off), yb = __shfl_up_sync(0xffffffffu, b, off);
        if (lane >= off) { a += ya; b += yb; }
      }
      b += __shfl_sync(0xffffffffu, a, 31);
      sm.gc[lane] = a;
      sm.gc[lane + 32] = b;
    }
    __syncthreads();
    const float glast = sm.gc[C - 1];
    if (threadIdx.x < C) {
      sm.eg[threadIdx.x] = expf(sm.gc[threadIdx.x]);
      sm.ed[threadIdx.x] = expf(glast - sm.gc[threadIdx.x]);
    }

    // ---- KK^T and QK^T (64 x 64): warp (wr, wc) rows 16 wr, cols 32 wc
    {
      float kk[4][4], qk[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) kk[j][e] = qk[j][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t ak[4], aq[4];
        frag_a(sm.ks, P16, 16 * wr, 16 * ks, ak);
        frag_a(sm.qs, P16, 16 * wr, 16 * ks, aq);
#pragma unroll
        for (int j2 = 0; j2 < 2; ++j2) {
          uint32_t b[4];
          frag_b_nk(sm.ks, P16, 32 * wc + 16 * j2, 16 * ks, b);
          mma(kk[2 * j2], ak, b[0], b[1]);
          mma(kk[2 * j2 + 1], ak, b[2], b[3]);
          mma(qk[2 * j2], aq, b[0], b[1]);
          mma(qk[2 * j2 + 1], aq, b[2], b[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 16 * wr + gr + (e >> 1) * 8;
          const int jj = 32 * wc + 8 * j + 2 * tq + (e & 1);
          const float decay = expf(fminf(sm.gc[i] - sm.gc[jj], 0.f));
          sm.amat[i * PF + jj] = i > jj ? -sm.beta[i] * kk[j][e] * decay : 0.f;
          sm.ps[i * P64 + jj] = __float2bfloat16_rn(i >= jj ? qk[j][e] * decay : 0.f);
        }
    }
    __syncthreads();
    // ---- T = (I - A)^-1 diagonal 16 x 16 blocks (warps 0-1: thread = block b, column j, column substitution), while
    // warps 2-7 make the scaled operand copies (the raw K and V are no longer needed after this)
    if (threadIdx.x < 64) {
      const int b = threadIdx.x >> 4, j = threadIdx.x & 15;
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
            if (m < i) acc += sm.amat[(base + i) * PF + base + m] * col[m];
          col[i] = acc;
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) sm.tf[(base + i) * PF + base + j] = col[i];
    } else {
      for (int i = threadIdx.x - 64; i < C * D / 2; i += 192) {
        const int t = i / (D / 2), d = (i % (D / 2)) * 2;
        const float eg = sm.eg[t], bt = sm.beta[t], ed = sm.ed[t];
        const float k0 = __bfloat162float(sm.ks[t * P16 + d]), k1 = __bfloat162float(sm.ks[t * P16 + d + 1]);
        const float q0 = __bfloat162float(sm.qs[t * P16 + d]), q1 = __bfloat162float(sm.qs[t * P16 + d + 1]);
        const float v0 = __bfloat162float(sm.vs[t * P16 + d]), v1 = __bfloat162float(sm.vs[t * P16 + d + 1]);
        *reinterpret_cast<uint32_t*>(&sm.kb[t * P16 + d]) = pack_bf2(k0 * bt * eg, k1 * bt * eg);
        *reinterpret_cast<uint32_t*>(&sm.kd[t * P16 + d]) = pack_bf2(k0 * ed, k1 * ed);
        *reinterpret_cast<uint32_t*>(&sm.qs[t * P16 + d]) = pack_bf2(q0 * eg, q1 * eg);
        *reinterpret_cast<uint32_t*>(&sm.vs[t * P16 + d]) = pack_bf2(v0 * bt, v1 * bt);
      }
    }
    __syncthreads();
    // off-diagonal blocks T_rc = T_rr (sum_{m=c}^{r-1} A_rm T_mc), by distance d = r - c from the diagonal: the
    // blocks of one distance need only blocks nearer the diagonal, so each distance is one parallel step. Thread =
    // (block c of the step, row i, 4 adjacent columns 4 q .. 4 q + 3): one load of A and one 16-byte load of T feed
    // four independent sums, each summed in the same order as an element-by-element loop.
    {
      const int bc = threadIdx.x >> 6, i = (threadIdx.x >> 2) & 15, q4 = (threadIdx.x & 3) * 4;
      for (int d = 1; d < 4; ++d) {
        const int c = bc, r = c + d;
        const bool active = c + d < 4;
        if (active) {
          float4 tmp = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int m = c; m < r; ++m)
#pragma unroll
            for (int kx = 0; kx < 16; ++kx) {
              const float av = sm.amat[(16 * r + i) * PF + 16 * m + kx];
              const float4 tv = *reinterpret_cast<const float4*>(&sm.tf[(16 * m + kx) * PF + 16 * c + q4]);
              tmp.x += av * tv.x;
              tmp.y += av * tv.y;
              tmp.z += av * tv.z;
              tmp.w += av * tv.w;
            }
          // staged in block (c, r) of amat's strictly upper part, which holds nothing
          *reinterpret_cast<float4*>(&sm.amat[(16 * c + i) * PF + 16 * r + q4]) = tmp;
        }
        __syncthreads();
        if (active) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int kx = 0; kx < 16; ++kx) {
            const float tv = sm.tf[(16 * r + i) * PF + 16 * r + kx];
            const float4 av = *reinterpret_cast<const float4*>(&sm.amat[(16 * c + kx) * PF + 16 * r + q4]);
            acc.x += tv * av.x;
            acc.y += tv * av.y;
            acc.z += tv * av.z;
            acc.w += tv * av.w;
          }
          *reinterpret_cast<float4*>(&sm.tf[(16 * r + i) * PF + 16 * c + q4]) = acc;
        }
        __syncthreads();
      }
    }
    // T (bf16), zero above the diagonal
    for (int idx = threadIdx.x; idx < C * C; idx += 256) {
      const int i = idx / C, j = idx % C;
      sm.ts[i * P64 + j] = __float2bfloat16_rn(j <= i ? sm.tf[i * PF + j] : 0.f);
    }
    __syncthreads();

    // ---- W = T (β e^gc K), then U = T (β V): warp rows 16 wr, cols 64 wc (8 n-blocks)
    float u[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) u[j][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < C / 16; ++ks) {
      uint32_t a[4];
      frag_a(sm.ts, P64, 16 * wr, 16 * ks, a);
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bk[4];
        frag_b_kn(sm.kb, P16, 64 * wc + 16 * j2, 16 * ks, bk);
        mma(u[2 * j2], a, bk[0], bk[1]);
        mma(u[2 * j2 + 1], a, bk[2], bk[3]);
      }
    }
    // W (bf16) over the raw K tile (free now)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r0 = 16 * wr + gr, cc = 64 * wc + 8 * j + 2 * tq;
      *reinterpret_cast<uint32_t*>(&sm.ks[r0 * P16 + cc]) = pack_bf2(u[j][0], u[j][1]);
      *reinterpret_cast<uint32_t*>(&sm.ks[(r0 + 8) * P16 + cc]) = pack_bf2(u[j][2], u[j][3]);
#pragma unroll
      for (int e = 0; e < 4; ++e) u[j][e] = 0.f;
    }
#pragma unroll
    for (int ks = 0; ks < C / 16; ++ks) {
      uint32_t a[4];
      frag_a(sm.ts, P64, 16 * wr, 16 * ks, a);
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bv[4];
        frag_b_kn(sm.vs, P16, 64 * wc + 16 * j2, 16 * ks, bv);
        mma(u[2 * j2], a, bv[0], bv[1]);
        mma(u[2 * j2 + 1], a, bv[2], bv[3]);
      }
    }
    __syncthreads();
    // ---- V' = U - W S  (k = 128 key dims), stored bf16 over β e^gc K (free now)
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a[4];
      frag_a(sm.ks, P16, 16 * wr, 16 * ks, a);
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t b[4];
        frag_b_kn(sm.sb, P16, 64 * wc + 16 * j2, 16 * ks, b);
        // accumulate -W S into u: negate by subtracting the product computed into a zero tile
        float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
        mma(t0, a, b[0], b[1]);
        mma(t1, a, b[2], b[3]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          u[2 * j2][e] -= t0[e];
          u[2 * j2 + 1][e] -= t1[e];
        }
      }
    }
    __syncthreads();   // everyone is done reading kb (as the W operand source) before it becomes V'
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r0 = 16 * wr + gr, cc = 64 * wc + 8 * j + 2 * tq;
      *reinterpret_cast<uint32_t*>(&sm.kb[r0 * P16 + cc]) = pack_bf2(u[j][0], u[j][1]);
      *reinterpret_cast<uint32_t*>(&sm.kb[(r0 + 8) * P16 + cc]) = pack_bf2(u[j][2], u[j][3]);
    }
    __syncthreads();
    // ---- O = scale ((e^gc Q) S + P V')
    {
      float acc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t a[4];
        frag_a(sm.qs, P16, 16 * wr, 16 * ks, a);
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t b[4];
          frag_b_kn(sm.sb, P16, 64 * wc + 16 * j2, 16 * ks, b);
          mma(acc[2 * j2], a, b[0], b[1]);
          mma(acc[2 * j2 + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        uint32_t a[4];
        frag_a(sm.ps, P64, 16 * wr, 16 * ks, a);
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t b[4];
          frag_b_kn(sm.kb, P16, 64 * wc + 16 * j2, 16 * ks, b);
          mma(acc[2 * j2], a, b[0], b[1]);
          mma(acc[2 * j2 + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int t0 = 16 * wr + gr, cc = 64 * wc + 8 * j + 2 * tq;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int t = t0 + 8 * hf;
          if (t < len) {
            const size_t tok = (size_t)row * n + c0 + t;
            const bool live = c0 + t < stop;
            *reinterpret_cast<uint32_t*>(o + (tok * NH + h) * D + cc) =
                live ? pack_bf2(acc[j][2 * hf] * scale, acc[j][2 * hf + 1] * scale) : 0u;
          }
        }
      }
    }
    __syncthreads();   // every read of ks / qs / vs / ps of this chunk is done
    if (c0 + C < n) issue_loads(c0 + C);   // the next chunk's tiles load during the state update
    // ---- S <- e^{gc_last} S + (e^{gc_last - gc} K)^T V'   (warp w: key rows 16w)
    const float el = expf(glast);
#pragma unroll
    for (int nb = 0; nb < 16; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nb][e] *= el;
#pragma unroll
    for (int ks = 0; ks < C / 16; ++ks) {
      uint32_t a[4];
      frag_a_t(sm.kd, P16, 16 * warp, 16 * ks, a);
#pragma unroll
      for (int j2 = 0; j2 < 8; ++j2) {
        uint32_t b[4];
        frag_b_kn(sm.kb, P16, 16 * j2, 16 * ks, b);
        mma(s[2 * j2], a, b[0], b[1]);
        mma(s[2 * j2 + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();   // all reads of this chunk's tiles are done before the next chunk overwrites them
  }
  if (out_tables) {
    const int opage = out_tables[(size_t)row * out_table_stride + flat / heads_per_page];
    float* s_out = reinterpret_cast<float*>(pool + (int64_t)opage * page_bytes + (flat % heads_per_page) * STATE_BYTES);
    const int r0 = 16 * warp + gr;
#pragma unroll
    for (int nb = 0; nb < 16; ++nb) {
      *reinterpret_cast<float2*>(s_out + (size_t)r0 * D + nb * 8 + 2 * tq) = make_float2(s[nb][0], s[nb][1]);
      *reinterpret_cast<float2*>(s_out + (size_t)(r0 + 8) * D + nb * 8 + 2 * tq) = make_float2(s[nb][2], s[nb][3]);
    }
  }
}

}  // namespace gdnc
}  // namespace jb

using namespace jb;

extern "C" int jb_gdn_scan(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                           const uint16_t* beta, uint16_t* o, int b, int n, void* pool, int64_t page_bytes,
                           const int32_t* tables, int table_stride, int first_head, int heads_per_page,
                           const int32_t* last, const int32_t* out_tables, int out_table_stride, void* stream) {
  JB_REQUIRE(q && k && v && g && beta && o && pool && tables, "jb_gdn_scan: null pointer");
  JB_REQUIRE(b > 0 && n > 0, "jb_gdn_scan: b %d, n %d", b, n);
  JB_REQUIRE(heads_per_page > 0 && (int64_t)heads_per_page * (int64_t)gdnc::STATE_BYTES <= page_bytes,
             "jb_gdn_scan: %d heads per page do not fit pages of %lld bytes", heads_per_page, (long long)page_bytes);
  JB_REQUIRE(first_head >= 0 && (first_head + gdnc::NH - 1) / heads_per_page < table_stride,
             "jb_gdn_scan: heads %d.. reach past the block table (%d entries)", first_head, table_stride);
  constexpr int SMEM = (int)sizeof(gdnc::Smem);
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    int r = status_of(cudaFuncSetAttribute(gdnc::chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM),
                      "gdn chunk: cudaFuncSetAttribute");
    if (r) return r;
    configured[dev] = true;
  }
  gdnc::chunk_kernel<<<b * gdnc::NH, 256, SMEM, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
      reinterpret_cast<const __nv_bfloat16*>(v), g, reinterpret_cast<const __nv_bfloat16*>(beta),
      reinterpret_cast<__nv_bfloat16*>(o), n, static_cast<uint8_t*>(pool), page_bytes, tables, table_stride,
      first_head, heads_per_page, last, out_tables, out_table_stride);
  return check_launch("gdn chunk_kernel");
}
