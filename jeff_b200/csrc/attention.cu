// S3 (first form): the attention input side, paged prefix-KV gated attention and the prefix pass's page scatter.
//
// Attention: one CTA per (row, key/value head, 16 new tokens) with 8 warps; warp w serves query head 4 g + (w & 3)
// and output dims [128 (w >> 2), +128). Keys come in tiles of 32 (one pool page of the prefix, then the row's own new
// keys), double-buffered in shared memory with cp.async; S = Q K^T and O += P V on bf16 mma.sync tensor-core tiles,
// an online softmax in fp32 (exp2, scale folded), P rounded to bf16 before the value product as the reference does
// (batched_kernels.py:405-427). Keys past the prefix length and future new keys are masked; their rows are zero-filled
// so stale page contents are never read into the sums.

namespace jb {
namespace attn {

constexpr int NQ = 8, NKV = 2, HD = 256, ROT = 64, PAGE = 32;
constexpr int BQ = 16;                 // new tokens per CTA
constexpr int BKN = 32;                // keys per tile
constexpr int PITCH = HD * 2 + 16;     // bytes per key row in shared memory (16 B pad: conflict-free)
constexpr int TILE_BYTES = BKN * PITCH;
constexpr int XCH_BYTES = 8 * 32 * 16 * 4;   // per warp, its partial S (16 x 32 fp32) for the warp sharing its head
constexpr int ATTN_SMEM = 4 * TILE_BYTES + XCH_BYTES;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// grid t, 12 warps: warps 0-7 query heads, 8-9 key heads, 10-11 value heads; lane = 8 dims
__global__ void __launch_bounds__(384) prep_kernel(const __nv_bfloat16* __restrict__ pr, int ldpr, int n,
                                                   const float* __restrict__ q_w1, const float* __restrict__ k_w1,
                                                   const float* __restrict__ inv_freq, const int* __restrict__ pos,
                                                   __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ kn,
                                                   __nv_bfloat16* __restrict__ vn) {
  pdl_begin();
  const int t = blockIdx.x;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = t / n;
  const __nv_bfloat16* src = pr + (size_t)t * ldpr;
  // the token's 32 rotary angles, shared by every query and key head: cos and sin rounded to bf16 once
  __shared__ float rc[ROT / 2], rsn[ROT / 2];
  if (threadIdx.x < ROT / 2) {
    const float f = (float)(pos[row] + (t - row * n)) * inv_freq[threadIdx.x];
    rc[threadIdx.x] = round_bf(cosf(f));
    rsn[threadIdx.x] = round_bf(sinf(f));
  }
  __syncthreads();
  if (w >= NQ + NKV) {
    const int hh = w - NQ - NKV;
    const uint4 val = reinterpret_cast<const uint4*>(src + NQ * 2 * HD + NKV * HD + hh * HD)[lane];
    reinterpret_cast<uint4*>(vn + ((size_t)t * NKV + hh) * HD)[lane] = val;
    return;
  }
  const bool is_q = w < NQ;
  const int base = is_q ? w * 2 * HD : NQ * 2 * HD + (w - NQ) * HD;
  const float* W = is_q ? q_w1 : k_w1;
  float x[8], y[8];
  const uint4 xu = reinterpret_cast<const uint4*>(src + base)[lane];
  x[0] = bf_lo(xu.x); x[1] = bf_hi(xu.x); x[2] = bf_lo(xu.y); x[3] = bf_hi(xu.y);
  x[4] = bf_lo(xu.z); x[5] = bf_hi(xu.z); x[6] = bf_lo(xu.w); x[7] = bf_hi(xu.w);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss += x[e] * x[e];
  const float rs = rsqrtf(warp_sum(ss) / HD + 1e-6f);
#pragma unroll
  for (int e = 0; e < 8; ++e) y[e] = round_bf(x[e] * rs * W[lane * 8 + e]);
  // lanes 0..7 hold dims 0..63: the rotate_half partner of dim d (< 32) is d + 32, four lanes up
  float part[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) part[e] = __shfl_xor_sync(0xffffffffu, y[e], 4);
  float out[8];
  if (lane < ROT / 8) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int d = lane * 8 + e;
      const float c = rc[d % (ROT / 2)], s = rsn[d % (ROT / 2)];
      const float rot = d < ROT / 2 ? -part[e] : part[e];
      out[e] = round_bf(y[e] * c) + round_bf(rot * s);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = y[e];
  }
  const uint4 ov = make_uint4(pack_bf2(out[0], out[1]), pack_bf2(out[2], out[3]), pack_bf2(out[4], out[5]),
                              pack_bf2(out[6], out[7]));
  if (is_q) reinterpret_cast<uint4*>(q + ((size_t)t * NQ + w) * HD)[lane] = ov;
  else reinterpret_cast<uint4*>(kn + ((size_t)t * NKV + (w - NQ)) * HD)[lane] = ov;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

struct Tile {
  int kind;   // 0 prefix page, 1 new keys
  int idx;    // page index in the prefix, or first new key
};

__global__ void __launch_bounds__(256, 1) paged_attention_kernel(
    const __nv_bfloat16* __restrict__ q, const uint8_t* __restrict__ pool, int64_t page_bytes,
    const int* __restrict__ tables, int table_stride, int kv_entry, int attn_layer, int attn_layers,
    const int* __restrict__ pos, const __nv_bfloat16* __restrict__ kn, const __nv_bfloat16* __restrict__ vn,
    __nv_bfloat16* __restrict__ out, int n, float scale_log2) {
  pdl_begin();
  extern __shared__ __align__(16) uint8_t sm[];
  // [buffer 0: K tile, V tile][buffer 1: K tile, V tile]
  const int row = blockIdx.x / NKV, g = blockIdx.x % NKV;
  const int qb = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = g * (NQ / NKV) + (warp & 3);
  const int dim0 = (warp >> 2) * 128;
  const int gr = lane >> 2, tq = lane & 3;
  const int P = pos[row];
  const int npages = (P + PAGE - 1) / PAGE;
  const int q_hi = (qb + 1) * BQ;                 // new keys this block may see: [0, q_hi)
  const int nnew = (q_hi + BKN - 1) / BKN;
  const int ntiles = npages + nnew;
  const int64_t layer_off = (int64_t)attn_layer * 2 * PAGE * NKV * HD * 2;
  const int64_t kv_half = (int64_t)PAGE * NKV * HD * 2;   // K block -> V block of one layer

  // Q fragments of this warp's half of the head dims [dim0, dim0 + 128): rows = tokens qb*16 + gr (+8). The warp
  // w ^ 4 holds the other half of the same head: each computes its half of Q K^T and they add the halves.
  uint32_t qf[8][4];
  {
    const size_t t0 = (size_t)row * n + qb * BQ + gr;
    const __nv_bfloat16* q0 = q + (t0 * NQ + head) * HD + dim0;
    const __nv_bfloat16* q1 = q + ((t0 + 8) * NQ + head) * HD + dim0;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qf[kk][0] = *reinterpret_cast<const uint32_t*>(q0 + kk * 16 + 2 * tq);
      qf[kk][1] = *reinterpret_cast<const uint32_t*>(q1 + kk * 16 + 2 * tq);
      qf[kk][2] = *reinterpret_cast<const uint32_t*>(q0 + kk * 16 + 8 + 2 * tq);
      qf[kk][3] = *reinterpret_cast<const uint32_t*>(q1 + kk * 16 + 8 + 2 * tq);
    }
  }
  float* xch = reinterpret_cast<float*>(sm + 4 * TILE_BYTES);   // [warp][16 values][32 lanes]
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -1e30f, m1 = -1e30f, l0 = 0.f, l1 = 0.f;

  auto load_tile = [&](int ti, int buf) {
    uint8_t* kd = sm + buf * 2 * TILE_BYTES;
    uint8_t* vd = kd + TILE_BYTES;
    // 32 keys x 512 B for K and for V: 2048 chunks of 16 B over 256 threads
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int idx = threadIdx.x + c * 256;
      const int kv = idx >> 10;            // 0 K, 1 V
      const int key = (idx >> 5) & 31;
      const int ch = idx & 31;
      const uint8_t* src;
      bool valid;
      if (ti < npages) {
        const int j = ti * PAGE + key;
        valid = j < P;
        const int page = tables[(size_t)row * table_stride + kv_entry + ti];
        src = pool + (int64_t)page * page_bytes + layer_off + kv * kv_half + ((int64_t)key * NKV + g) * HD * 2 + ch * 16;
      } else {
        const int kk = (ti - npages) * BKN + key;
        valid = kk < q_hi;
        const __nv_bfloat16* base = kv ? vn : kn;
        src = reinterpret_cast<const uint8_t*>(base + (((size_t)row * n + (valid ? kk : 0)) * NKV + g) * HD) + ch * 16;
      }
      if (!valid) src = reinterpret_cast<const uint8_t*>(kn);
      cp_async16(smem_u32((kv ? vd : kd) + key * PITCH + ch * 16), src, valid);
    }
    cp_async_commit();
  };

  if (ntiles > 0) load_tile(0, 0);
  for (int ti = 0; ti < ntiles; ++ti) {
    const int buf = ti & 1;
    if (ti + 1 < ntiles) {
      load_tile(ti + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint8_t* ks = sm + buf * 2 * TILE_BYTES;
    const uint8_t* vs = ks + TILE_BYTES;
    // S = Q K^T: 16 rows x 32 keys, this warp's 128 dims (K fragments by ldmatrix: keys as rows), then the
    // partner's partial added (a + b = b + a: both warps hold the same S)
    float s[4][4];
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
      const int mi = lane >> 3;
      const uint8_t* krow = ks + (nb * 8 + (lane & 7)) * PITCH + dim0 * 2 + (mi & 1) * 16 + (mi >> 1) * 32;
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(krow + kk * 32), b0, b1, b2, b3);
        mma16816(s[nb], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816(s[nb], qf[kk + 1][0], qf[kk + 1][1], qf[kk + 1][2], qf[kk + 1][3], b2, b3);
      }
    }
#pragma unroll
    for (int nb = 0; nb < 4; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) xch[(warp * 16 + nb * 4 + e) * 32 + lane] = s[nb][e];
    named_barrier(1 + (warp & 3), 64);   // the two warps of this head
#pragma unroll
    for (int nb = 0; nb < 4; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nb][e] += xch[((warp ^ 4) * 16 + nb * 4 + e) * 32 + lane];
    // masks and the online softmax (rows gr and gr + 8 of this warp)
    const int tok0 = qb * BQ + gr, tok1 = tok0 + 8;
    float mx0 = m0, mx1 = m1;
    bool ok[4][4];
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = nb * 8 + 2 * tq + (e & 1);
        bool valid;
        if (ti < npages) {
          valid = ti * PAGE + key < P;
        } else {
          const int kk = (ti - npages) * BKN + key;
          valid = kk <= (e < 2 ? tok0 : tok1);
        }
        ok[nb][e] = valid;
        s[nb][e] = valid ? s[nb][e] * scale_log2 : -1e30f;
      }
      mx0 = fmaxf(mx0, fmaxf(s[nb][0], s[nb][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nb][2], s[nb][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float al0 = exp2f(m0 - mx0), al1 = exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pf[4][2];
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      const float p0 = ok[nb][0] ? exp2f(s[nb][0] - mx0) : 0.f;
      const float p1 = ok[nb][1] ? exp2f(s[nb][1] - mx0) : 0.f;
      const float p2 = ok[nb][2] ? exp2f(s[nb][2] - mx1) : 0.f;
      const float p3 = ok[nb][3] ? exp2f(s[nb][3] - mx1) : 0.f;
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      pf[nb][0] = pack_bf2(p0, p1);
      pf[nb][1] = pack_bf2(p2, p3);
    }
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= al0;
      o[i][1] *= al0;
      o[i][2] *= al1;
      o[i][3] *= al1;
    }
    // O += P V: P (16 x 32 keys) as A in two k16 steps, V^T fragments by ldmatrix.trans
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const uint32_t a0 = pf[2 * kk][0], a1 = pf[2 * kk][1], a2 = pf[2 * kk + 1][0], a3 = pf[2 * kk + 1][1];
      const int mi = lane >> 3, r = lane & 7;
      const int key = kk * 16 + (mi & 1) * 8 + r;
#pragma unroll
      for (int nb2 = 0; nb2 < 8; ++nb2) {
        const int dim = dim0 + nb2 * 16 + (mi >> 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(smem_u32(vs + key * PITCH + dim * 2), b0, b1, b2, b3);
        mma16816(o[2 * nb2], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * nb2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }
  const float inv0 = l0 > 0.f ? 1.0f / l0 : 0.f, inv1 = l1 > 0.f ? 1.0f / l1 : 0.f;
  const size_t t0 = (size_t)row * n + qb * BQ + gr;
  __nv_bfloat16* o0p = out + (t0 * NQ + head) * HD + dim0;
  __nv_bfloat16* o1p = out + ((t0 + 8) * NQ + head) * HD + dim0;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int d = i * 8 + 2 * tq;
    *reinterpret_cast<uint32_t*>(o0p + d) = pack_bf2(o[i][0] * inv0, o[i][1] * inv0);
    *reinterpret_cast<uint32_t*>(o1p + d) = pack_bf2(o[i][2] * inv1, o[i][3] * inv1);
  }
}

// prefix pass: kn/vn of token j of row r into page out_tables[r][kv_entry + j / 32] (tokens below the row's last page)
__global__ void kv_scatter_kernel(const __nv_bfloat16* __restrict__ kn, const __nv_bfloat16* __restrict__ vn, int b,
                                  int n, const int* __restrict__ real, uint8_t* __restrict__ pool, int64_t page_bytes,
                                  const int* __restrict__ out_tables, int table_stride, int kv_entry, int attn_layer) {
  pdl_begin();
  constexpr int CH = NKV * HD * 2 / 16;   // 16-byte chunks per token per K or V
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)b * n * 2 * CH) return;
  const int c = (int)(i % CH);
  const int kv = (int)((i / CH) % 2);
  const size_t t = i / (2 * CH);
  const int row = (int)(t / n), j = (int)(t % n);
  const int kept = ((real[row] + PAGE - 1) / PAGE) * PAGE;
  if (j >= kept) return;
  const int page = out_tables[(size_t)row * table_stride + kv_entry + j / PAGE];
  const int64_t off = (int64_t)page * page_bytes + (int64_t)attn_layer * 2 * PAGE * NKV * HD * 2 +
                      (int64_t)kv * PAGE * NKV * HD * 2 + (int64_t)(j % PAGE) * NKV * HD * 2 + c * 16;
  const __nv_bfloat16* src = (kv ? vn : kn) + t * NKV * HD;
  *reinterpret_cast<uint4*>(pool + off) = reinterpret_cast<const uint4*>(src)[c];
}

}  // namespace attn
}  // namespace jb

using namespace jb;

extern "C" int jb_attn_prep_rows(const uint16_t* pr, int ldpr, int t, int n, const float* q_w1, const float* k_w1,
                                 const float* inv_freq, const int32_t* pos, uint16_t* q, uint16_t* kn, uint16_t* vn,
                                 void* stream) {
  JB_REQUIRE(pr && q_w1 && k_w1 && inv_freq && pos && q && kn && vn, "jb_attn_prep_rows: null pointer");
  JB_REQUIRE(t > 0 && n > 0 && t % n == 0, "jb_attn_prep_rows: a pass of %d tokens in rows of %d", t, n);
  JB_REQUIRE(ldpr >= attn::NQ * 2 * attn::HD + 2 * attn::NKV * attn::HD && ldpr % 8 == 0, "jb_attn_prep_rows: ldpr %d",
             ldpr);
  launch_pdl(attn::prep_kernel, t, 384, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(pr), ldpr, n, q_w1, k_w1, inv_freq, pos,
      reinterpret_cast<__nv_bfloat16*>(q), reinterpret_cast<__nv_bfloat16*>(kn), reinterpret_cast<__nv_bfloat16*>(vn));
  return check_launch("attn prep_kernel");
}

extern "C" int jb_paged_attention(const uint16_t* q, const void* pool, int64_t page_bytes, const int32_t* tables,
                                  int table_stride, int kv_entry, int attn_layer, int attn_layers, const int32_t* pos,
                                  const uint16_t* kn, const uint16_t* vn, uint16_t* out, int b, int n, void* stream) {
  JB_REQUIRE(q && pool && tables && pos && kn && vn && out, "jb_paged_attention: null pointer");
  JB_REQUIRE(b > 0 && n > 0 && n % attn::BQ == 0, "jb_paged_attention: b %d, n %d (a multiple of 16)", b, n);
  JB_REQUIRE(attn_layer >= 0 && attn_layer < attn_layers &&
                 (int64_t)attn_layers * 2 * attn::PAGE * attn::NKV * attn::HD * 2 <= page_bytes,
             "jb_paged_attention: attention layer %d of %d does not fit pages of %lld bytes", attn_layer, attn_layers,
             (long long)page_bytes);
  JB_REQUIRE(kv_entry >= 0 && kv_entry <= table_stride, "jb_paged_attention: kv_entry %d", kv_entry);
  constexpr int SMEM = attn::ATTN_SMEM;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    int r = status_of(cudaFuncSetAttribute(attn::paged_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           SMEM),
                      "paged_attention: cudaFuncSetAttribute");
    if (r) return r;
    configured[dev] = true;
  }
  dim3 grid(b * attn::NKV, n / attn::BQ);
  launch_pdl(attn::paged_attention_kernel, grid, 256, SMEM, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(q), static_cast<const uint8_t*>(pool), page_bytes, tables, table_stride,
      kv_entry, attn_layer, attn_layers, pos, reinterpret_cast<const __nv_bfloat16*>(kn),
      reinterpret_cast<const __nv_bfloat16*>(vn), reinterpret_cast<__nv_bfloat16*>(out), n,
      (1.0f / 16.0f) * 1.4426950408889634f);
  return check_launch("paged_attention_kernel");
}

extern "C" int jb_kv_scatter(const uint16_t* kn, const uint16_t* vn, int b, int n, const int32_t* real, void* pool,
                             int64_t page_bytes, const int32_t* out_tables, int table_stride, int kv_entry,
                             int attn_layer, int attn_layers, void* stream) {
  JB_REQUIRE(kn && vn && real && pool && out_tables, "jb_kv_scatter: null pointer");
  JB_REQUIRE(b > 0 && n > 0 && n % attn::PAGE == 0, "jb_kv_scatter: b %d, n %d (a multiple of 32)", b, n);
  JB_REQUIRE(kv_entry + n / attn::PAGE <= table_stride, "jb_kv_scatter: %d pages past entry %d exceed the table (%d)",
             n / attn::PAGE, kv_entry, table_stride);
  JB_REQUIRE(attn_layer >= 0 && attn_layer < attn_layers &&
                 (int64_t)attn_layers * 2 * attn::PAGE * attn::NKV * attn::HD * 2 <= page_bytes,
             "jb_kv_scatter: attention layer %d of %d", attn_layer, attn_layers);
  const size_t total = (size_t)b * n * 2 * (attn::NKV * attn::HD * 2 / 16);
  launch_pdl(attn::kv_scatter_kernel, (unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream,
      reinterpret_cast<const __nv_bfloat16*>(kn), reinterpret_cast<const __nv_bfloat16*>(vn), b, n, real,
      static_cast<uint8_t*>(pool), page_bytes, out_tables, table_stride, kv_entry, attn_layer);
  return check_launch("kv_scatter_kernel");
}
