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
constexpr int QKV_CH = 6144;                           // convolved channels q | k | v of the in_proj output
constexpr size_t CONV_TAIL_BYTES = (size_t)3 * QKV_CH * 2;   // a layer's cached conv inputs (3, 6144) bf16

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

// ---------------------------------------------------------------- one chunk of the rule (shared by both kernels)
//
// On entry: ks / qs / vs hold the chunk's K, Q, V tiles (bf16, zero past len), sm.gc each token's log-decay g and
// sm.beta its beta (both zero past len), s the state entering the chunk (fp32 accumulators, warp w: key rows 16w +
// gr (+8), value cols 8nb + 2tq (+1)). Computes O = scale ((e^gc Q) S + P V') and hands it to emit(acc) (every
// thread calls it; acc rows 16 wr + gr (+8), cols 64 wc + 8j + 2tq (+1) of the 64 x 128 tile, unscaled), then,
// after a barrier, calls before_update() (every read of ks / qs / vs / ps of this chunk is done by then) and folds
// the chunk into s.
template <class Emit, class BeforeUpdate>
__device__ __forceinline__ void chunk_step(Smem& sm, float (&s)[16][4], Emit&& emit, BeforeUpdate&& before_update) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gr = lane >> 2, tq = lane & 3;
  const int wr = warp & 3;          // 16-row block of the 64-row tiles this warp computes
  const int wc = warp >> 2;         // column half (64 of 128) of the 64 x 128 tiles
  // ---- S (bf16) for this chunk's operands
#pragma unroll
  for (int nb = 0; nb < 16; ++nb) {
    const int r0 = 16 * warp + gr, cc = nb * 8 + 2 * tq;
    *reinterpret_cast<uint32_t*>(&sm.sb[r0 * P16 + cc]) = pack_bf2(s[nb][0], s[nb][1]);
    *reinterpret_cast<uint32_t*>(&sm.sb[(r0 + 8) * P16 + cc]) = pack_bf2(s[nb][2], s[nb][3]);
  }
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
  // ---- O = (e^gc Q) S + P V'
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
    emit(acc);
  }
  __syncthreads();   // every read of ks / qs / vs / ps of this chunk is done
  before_update();
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

__device__ __forceinline__ const float* state_in(const uint8_t* pool, int64_t page_bytes, const int* tables,
                                                 int table_stride, int row, int flat, int heads_per_page) {
  const int page = tables[(size_t)row * table_stride + flat / heads_per_page];
  return reinterpret_cast<const float*>(pool + (int64_t)page * page_bytes + (flat % heads_per_page) * STATE_BYTES);
}

__device__ __forceinline__ void load_state(const float* s_in, float (&s)[16][4]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gr = lane >> 2, tq = lane & 3;
  const int r0 = 16 * warp + gr;
#pragma unroll
  for (int nb = 0; nb < 16; ++nb) {
    const float2 lo = *reinterpret_cast<const float2*>(s_in + (size_t)r0 * D + nb * 8 + 2 * tq);
    const float2 hi = *reinterpret_cast<const float2*>(s_in + (size_t)(r0 + 8) * D + nb * 8 + 2 * tq);
    s[nb][0] = lo.x; s[nb][1] = lo.y; s[nb][2] = hi.x; s[nb][3] = hi.y;
  }
}

__device__ __forceinline__ void store_state(float* s_out, const float (&s)[16][4]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gr = lane >> 2, tq = lane & 3;
  const int r0 = 16 * warp + gr;
#pragma unroll
  for (int nb = 0; nb < 16; ++nb) {
    *reinterpret_cast<float2*>(s_out + (size_t)r0 * D + nb * 8 + 2 * tq) = make_float2(s[nb][0], s[nb][1]);
    *reinterpret_cast<float2*>(s_out + (size_t)(r0 + 8) * D + nb * 8 + 2 * tq) = make_float2(s[nb][2], s[nb][3]);
  }
}

// ---------------------------------------------------------------- the rule alone (q, k, v, g, beta given)

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
  pdl_begin();
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

  float s[16][4];
  load_state(state_in(pool, page_bytes, tables, table_stride, row, flat, heads_per_page), s);
  const int wr = warp & 3, wc = warp >> 2;

  for (int c0 = 0; c0 < n; c0 += C) {
    const int len = min(C, n - c0);
    if (threadIdx.x < C) {
      const int t = threadIdx.x;
      const size_t tok = (size_t)row * n + c0 + t;
      sm.gc[t] = t < len ? g[tok * NH + h] : 0.f;
      sm.beta[t] = t < len ? __bfloat162float(beta[tok * NH + h]) : 0.f;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    chunk_step(
        sm, s,
        [&](float (&acc)[8][4]) {
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
        },
        [&]() {
          if (c0 + C < n) issue_loads(c0 + C);   // the next chunk's tiles load during the state update
        });
  }
  if (out_tables) {
    const int opage = out_tables[(size_t)row * out_table_stride + flat / heads_per_page];
    store_state(reinterpret_cast<float*>(pool + (int64_t)opage * page_bytes + (flat % heads_per_page) * STATE_BYTES),
                s);
  }
}

// ---------------------------------------------------------------- the whole Gated DeltaNet mixer of a layer
//
// One CTA (8 warps) per (row, head): the in_proj output pr (T, ldpr) = [q 2048 | k 2048 | v 2048 | z 2048 | b 16 |
// a 16] is read chunk by chunk by cp.async (this head's 128 raw q, k, v inputs into a staging area that the rule
// only uses during its T solve, its z columns and its b, a); then, in parallel over (token, part), the causal
// depthwise convolution over [3 cached inputs; the row's inputs] (fp32), SiLU rounded to bf16, and for q and k the
// L2 norm (eps 1e-6) by one warp per token (lane = 4 channels), written into the tiles the rule multiplies; the gates
// g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) (the reference's gdn_prep_rows, batched_kernels.py:89-194);
// then the chunked rule (chunk_step); then the gated RMSNorm y = bf16(bf16(w bf16(rms(o))) silu(z))
// (fast_path.py:103-120) of the chunk's bf16 outputs, written as y (T, ldy) bf16 columns [128 h, 128 h + 128).
// q, k, v, g, beta and o never leave the SM. Every value and rounding is the same as jb_gdn_prep_rows + jb_gdn_scan
// + jb_gated_norm in sequence, so y is bit-identical to theirs. The next chunk's inputs load while the state update
// of this one runs. Prefix pass (real and out_tables): tokens past real[row] get g = beta = 0, the row's last three
// real inputs of the head's channels go to its conv tail page and its final state to its state page.
constexpr int RAW = 3 * D;                  // raw conv inputs of a head: q | k | v channels

struct LayerSmem {
  Smem scan;                                // the raw q | k | v tiles of the next chunk are staged over amat .. ps
  __nv_bfloat16 zs[C * P16];                // the chunk's z columns of the head
  __nv_bfloat16 ba[C * 32];                 // the chunk's b (16) | a (16)
  __nv_bfloat16 hist[2][3 * RAW];           // raw inputs at positions c0 - 3 .. c0 - 1, by chunk parity
};
static_assert(3 * C * P16 * 2 <= sizeof(float) * 2 * C * PF + 2 * C * P64 * 2,
              "raw q | k | v tiles fit over amat, tf, ts and ps");

__global__ void __launch_bounds__(256, 1) layer_kernel(const __nv_bfloat16* __restrict__ pr, int ldpr, int n,
                                                       uint8_t* __restrict__ pool, int64_t page_bytes,
                                                       const int* __restrict__ tables, int table_stride,
                                                       int first_head, int heads_per_page, int conv_entry,
                                                       int conv_slot, const float* __restrict__ conv_w,
                                                       const float* __restrict__ a_neg,
                                                       const float* __restrict__ dt_bias,
                                                       const __nv_bfloat16* __restrict__ gnorm_w,
                                                       __nv_bfloat16* __restrict__ y, int ldy,
                                                       const int* __restrict__ last, const int* __restrict__ real,
                                                       const int* __restrict__ out_tables, int out_table_stride) {
  pdl_begin();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  LayerSmem& L = *reinterpret_cast<LayerSmem*>(smem_raw);
  Smem& sm = L.scan;
  // raw tiles: part p (0 q, 1 k, 2 v) at raw + p * C * P16, row t = token c0 + t
  __nv_bfloat16* raw = reinterpret_cast<__nv_bfloat16*>(sm.amat);
  const int row = blockIdx.x / NH, h = blockIdx.x % NH;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gr = lane >> 2, tq = lane & 3;
  const int wr = warp & 3, wc = warp >> 2;
  const int flat = first_head + h;
  const float scale = rsqrtf((float)D);
  const int stop = last ? min(last[row] + 1, n) : n;     // outputs past stop are those of o = 0
  const int rl = real ? real[row] : n;                    // tokens from rl on leave the state unchanged
  const size_t rbase = (size_t)row * n;

  auto issue_loads = [&](int c0) {
    const int len = min(C, n - c0);
    constexpr int PER_TOKEN = 4 * (D / 8) + 4;   // 16-byte pieces: q, k, v, z (16 each), b | a (4)
    for (int i = tid; i < C * PER_TOKEN; i += 256) {
      const int t = i / PER_TOKEN, piece = i % PER_TOKEN;
      const bool valid = t < len;
      const __nv_bfloat16* src = pr + (rbase + c0 + (valid ? t : 0)) * ldpr;
      __nv_bfloat16* dst;
      if (piece < 4 * (D / 8)) {
        const int part = piece >> 4, c8 = (piece & 15) * 8;     // part: 0 q, 1 k, 2 v, 3 z
        src += part * 2048 + h * D + c8;
        dst = (part < 3 ? raw + part * C * P16 : L.zs) + t * P16 + c8;
      } else {
        const int c8 = (piece - 4 * (D / 8)) * 8;
        src += 4 * 2048 + c8;
        dst = L.ba + t * 32 + c8;
      }
      cp_async16(dst, src, valid);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue_loads(0);

  // chunk 0's cached inputs: the layer's conv tail page of the row, this head's q | k | v channels
  {
    const int page = tables[(size_t)row * table_stride + conv_entry];
    const __nv_bfloat16* tail =
        reinterpret_cast<const __nv_bfloat16*>(pool + (int64_t)page * page_bytes + conv_slot * CONV_TAIL_BYTES);
    for (int i = tid; i < 3 * RAW / 8; i += 256) {
      const int r = i / (RAW / 8), c8 = (i % (RAW / 8)) * 8;
      *reinterpret_cast<uint4*>(&L.hist[0][r * RAW + c8]) =
          *reinterpret_cast<const uint4*>(tail + (size_t)r * QKV_CH + (c8 / D) * 2048 + h * D + c8 % D);
    }
  }
  float s[16][4];
  load_state(state_in(pool, page_bytes, tables, table_stride, row, flat, heads_per_page), s);

  int parity = 0;
  for (int c0 = 0; c0 < n; c0 += C, parity ^= 1) {
    const int len = min(C, n - c0);
    const __nv_bfloat16* hist = L.hist[parity];
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // raw input at chunk position t (-3 <= t < C) of channel c (0..383) of the head
    auto raw_at = [&](int t, int c) -> const __nv_bfloat16* {
      return t >= 0 ? raw + (c / D) * C * P16 + t * P16 + c % D : hist + (t + 3) * RAW + c;
    };
    if (real && out_tables && ((c0 <= rl - 1 && rl - 1 < c0 + C) || (rl <= 0 && c0 == 0))) {
      // the prefix pass: the row's last three real inputs become its cached tail
      const int opage = out_tables[(size_t)row * out_table_stride + conv_entry];
      __nv_bfloat16* otail =
          reinterpret_cast<__nv_bfloat16*>(pool + (int64_t)opage * page_bytes + conv_slot * CONV_TAIL_BYTES);
      for (int i = tid; i < 3 * RAW / 8; i += 256) {
        const int r = i / (RAW / 8), c8 = (i % (RAW / 8)) * 8;
        *reinterpret_cast<uint4*>(otail + (size_t)r * QKV_CH + (c8 / D) * 2048 + h * D + c8 % D) =
            *reinterpret_cast<const uint4*>(raw_at(rl - 3 + r - c0, c8));
      }
    }
    if (tid < C) {   // gates of the chunk's tokens
      const int t = tid;
      float gv = 0.f, bt = 0.f;
      if (t < len && c0 + t < rl) {
        const float bv = __bfloat162float(L.ba[t * 32 + h]);
        const float av = __bfloat162float(L.ba[t * 32 + NH + h]) + dt_bias[h];
        const float sp = av > 20.0f ? av : logf(1.0f + expf(av));
        gv = a_neg[h] * sp;
        bt = round_bf(1.0f / (1.0f + expf(-bv)));
      }
      sm.gc[t] = gv;
      sm.beta[t] = bt;
    }
    // conv + SiLU (+ the L2 norm for q and k): warp = one (token, part) at a time, lane = 4 channels
#pragma unroll
    for (int part = 0; part < 3; ++part) {
      float taps[4][4];   // this lane's channels 4 lane .. + 3 of the part
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 wv =
            *reinterpret_cast<const float4*>(conv_w + (size_t)i * QKV_CH + part * 2048 + h * D + 4 * lane);
        taps[i][0] = wv.x;
        taps[i][1] = wv.y;
        taps[i][2] = wv.z;
        taps[i][3] = wv.w;
      }
      __nv_bfloat16* tile = part == 0 ? sm.qs : part == 1 ? sm.ks : sm.vs;
      const int c = part * D + 4 * lane;
#pragma unroll 2
      for (int t = warp; t < C; t += 8) {
        float x[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint2 u = *reinterpret_cast<const uint2*>(raw_at(t - 3 + j, c));
          x[j][0] = bf_lo(u.x);
          x[j][1] = bf_hi(u.x);
          x[j][2] = bf_lo(u.y);
          x[j][3] = bf_hi(u.y);
        }
        float cv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float acc = 0.f;
          acc += taps[0][e] * x[0][e];
          acc += taps[1][e] * x[1][e];
          acc += taps[2][e] * x[2][e];
          acc += taps[3][e] * x[3][e];
          // SiLU with the fast intrinsics, rounded to bf16 at once (as jb_gdn_prep_rows)
          cv[e] = t < len ? round_bf(__fdividef(acc, 1.0f + __expf(-acc))) : 0.f;
        }
        if (part < 2) {
          float ss = cv[0] * cv[0] + cv[1] * cv[1] + cv[2] * cv[2] + cv[3] * cv[3];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          const float rs = rsqrtf(ss + 1e-6f);
#pragma unroll
          for (int e = 0; e < 4; ++e) cv[e] *= rs;
        }
        *reinterpret_cast<uint2*>(&tile[t * P16 + 4 * lane]) =
            make_uint2(pack_bf2(cv[0], cv[1]), pack_bf2(cv[2], cv[3]));
      }
    }
    // the next chunk's cached inputs: this chunk's last three raw rows (the other parity's buffer)
    if (c0 + C < n)
      for (int i = tid; i < 3 * RAW / 8; i += 256) {
        const int r = i / (RAW / 8), c8 = (i % (RAW / 8)) * 8;
        *reinterpret_cast<uint4*>(&L.hist[parity ^ 1][r * RAW + c8]) =
            *reinterpret_cast<const uint4*>(raw_at(C - 3 + r, c8));
      }
    __syncthreads();
    chunk_step(
        sm, s,
        [&](float (&acc)[8][4]) {
          // the chunk's bf16 outputs (zero past stop) into vs, free since U was formed
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int ccol = 64 * wc + 8 * j + 2 * tq;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              const int t = 16 * wr + gr + 8 * hf;
              const bool live = c0 + t < stop;
              *reinterpret_cast<uint32_t*>(&sm.vs[t * P16 + ccol]) =
                  live ? pack_bf2(acc[j][2 * hf] * scale, acc[j][2 * hf + 1] * scale) : 0u;
            }
          }
          __syncthreads();
          // gated RMSNorm: 16 threads per token, 8 consecutive values each (as jb_gated_norm)
#pragma unroll
          for (int task = tid; task < C * 16; task += 256) {
            const int t = task >> 4, sub = task & 15;
            const uint4 ov = *reinterpret_cast<const uint4*>(&sm.vs[t * P16 + 8 * sub]);
            const uint4 zv = *reinterpret_cast<const uint4*>(&L.zs[t * P16 + 8 * sub]);
            const uint4 wv = *reinterpret_cast<const uint4*>(gnorm_w + 8 * sub);
            const float v8[8] = {bf_lo(ov.x), bf_hi(ov.x), bf_lo(ov.y), bf_hi(ov.y),
                                 bf_lo(ov.z), bf_hi(ov.z), bf_lo(ov.w), bf_hi(ov.w)};
            const float z8[8] = {bf_lo(zv.x), bf_hi(zv.x), bf_lo(zv.y), bf_hi(zv.y),
                                 bf_lo(zv.z), bf_hi(zv.z), bf_lo(zv.w), bf_hi(zv.w)};
            const float w8[8] = {bf_lo(wv.x), bf_hi(wv.x), bf_lo(wv.y), bf_hi(wv.y),
                                 bf_lo(wv.z), bf_hi(wv.z), bf_lo(wv.w), bf_hi(wv.w)};
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) ss += v8[e] * v8[e];
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            const float rs = rsqrtf(ss / 128.f + 1e-6f);
            float out[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float nv = round_bf(v8[e] * rs);
              const float gw = round_bf(w8[e] * nv);
              out[e] = gw * (z8[e] / (1.0f + expf(-z8[e])));
            }
            if (t < len)
              *reinterpret_cast<uint4*>(y + (rbase + c0 + t) * ldy + h * D + 8 * sub) =
                  make_uint4(pack_bf2(out[0], out[1]), pack_bf2(out[2], out[3]), pack_bf2(out[4], out[5]),
                             pack_bf2(out[6], out[7]));
          }
        },
        [&]() {
          if (c0 + C < n) issue_loads(c0 + C);   // the next chunk's inputs load during the state update
        });
  }
  if (out_tables) {
    const int opage = out_tables[(size_t)row * out_table_stride + flat / heads_per_page];
    store_state(reinterpret_cast<float*>(pool + (int64_t)opage * page_bytes + (flat % heads_per_page) * STATE_BYTES),
                s);
  }
}

// The dynamic shared memory attribute of a kernel, set on every launch: the attribute belongs to the current device
// and setting it costs a driver call of well under a microsecond, so no per-device cache (and no race between host
// threads over one) is needed.
template <class Kernel>
int configure(Kernel kernel, int smem_bytes, const char* what) {
  return status_of(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes), what);
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
  int st = gdnc::configure(gdnc::chunk_kernel, SMEM, "gdn chunk_kernel");
  if (st) return st;
  launch_pdl(gdnc::chunk_kernel, b * gdnc::NH, 256, SMEM, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
      reinterpret_cast<const __nv_bfloat16*>(v), g, reinterpret_cast<const __nv_bfloat16*>(beta),
      reinterpret_cast<__nv_bfloat16*>(o), n, static_cast<uint8_t*>(pool), page_bytes, tables, table_stride,
      first_head, heads_per_page, last, out_tables, out_table_stride);
  return check_launch("gdn chunk_kernel");
}

extern "C" int jb_gdn_layer(const uint16_t* pr, int ldpr, int t, int n, void* pool, int64_t page_bytes,
                            const int32_t* tables, int table_stride, int first_head, int heads_per_page,
                            int conv_entry, int conv_slot, const float* conv_w, const float* a_neg,
                            const float* dt_bias, const uint16_t* gnorm_w, uint16_t* y, int ldy, const int32_t* last,
                            const int32_t* real, const int32_t* out_tables, int out_table_stride, void* stream) {
  JB_REQUIRE(pr && pool && tables && conv_w && a_neg && dt_bias && gnorm_w && y, "jb_gdn_layer: null pointer");
  JB_REQUIRE(t > 0 && n > 0 && t % n == 0, "jb_gdn_layer: a pass of %d tokens in rows of %d", t, n);
  JB_REQUIRE(ldpr >= 4 * 2048 + 32 && ldpr % 8 == 0, "jb_gdn_layer: ldpr %d (>= 8224, a multiple of 8)", ldpr);
  JB_REQUIRE(ldy >= gdnc::NH * gdnc::D && ldy % 8 == 0, "jb_gdn_layer: ldy %d (>= 2048, a multiple of 8)", ldy);
  JB_REQUIRE(((reinterpret_cast<uintptr_t>(pr) | reinterpret_cast<uintptr_t>(y) |
               reinterpret_cast<uintptr_t>(gnorm_w) | reinterpret_cast<uintptr_t>(conv_w)) & 15) == 0,
             "jb_gdn_layer: pr, y, gnorm_w and conv_w must be 16-byte aligned");
  JB_REQUIRE(heads_per_page > 0 && (int64_t)heads_per_page * (int64_t)gdnc::STATE_BYTES <= page_bytes,
             "jb_gdn_layer: %d heads per page do not fit pages of %lld bytes", heads_per_page, (long long)page_bytes);
  JB_REQUIRE(first_head >= 0 && (first_head + gdnc::NH - 1) / heads_per_page < table_stride,
             "jb_gdn_layer: heads %d.. reach past the block table (%d entries)", first_head, table_stride);
  JB_REQUIRE(conv_entry >= 0 && conv_entry < table_stride && conv_slot >= 0 &&
                 (int64_t)(conv_slot + 1) * (int64_t)gdnc::CONV_TAIL_BYTES <= page_bytes,
             "jb_gdn_layer: conv entry %d / slot %d do not fit the page geometry", conv_entry, conv_slot);
  JB_REQUIRE(!out_tables || (real && out_table_stride > 0), "jb_gdn_layer: out_tables needs real and its stride");
  constexpr int SMEM = (int)sizeof(gdnc::LayerSmem);
  static_assert(SMEM <= 227 * 1024, "shared memory");
  int st = gdnc::configure(gdnc::layer_kernel, SMEM, "gdn layer_kernel");
  if (st) return st;
  launch_pdl(gdnc::layer_kernel, (t / n) * gdnc::NH, 256, SMEM, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(pr), ldpr, n, static_cast<uint8_t*>(pool), page_bytes, tables,
      table_stride, first_head, heads_per_page, conv_entry, conv_slot, conv_w, a_neg, dt_bias,
      reinterpret_cast<const __nv_bfloat16*>(gnorm_w), reinterpret_cast<__nv_bfloat16*>(y), ldy, last, real,
      out_tables, out_table_stride);
  return check_launch("gdn layer_kernel");
}
