// Dense transforms and elementwise ops with the reference's rounding.
//
// X*W (wasmMatmul, src/backend/wasm/index.ts:18-63): for every output (i,j)
// the reference runs k = 0..K-1 in ascending order and stores
// f32(acc + a*b) (double arithmetic) after each step.  The kernel keeps that
// order: each output is owned by one thread that walks k ascending.
//   BGNN_MATH_EXACT: f64 fma (the product of two floats is exact in double)
//                    then one rounding to f32 -- the reference's bits.
//   BGNN_MATH_FAST:  f32 fma in the same order (packed two per instruction);
//                    differs from the reference only where its double result
//                    lands on an f32 tie.
// K tails are not zero-padded (an extra fma with 0 could turn a -0 into +0).
// SAGE stores f32(self + neigh) (Tensor.add -> wasmAdd, sage.ts:178-183):
// the kernel runs twice, storing St = X*W_self as f32 (as the reference's
// Tensor does) and adding it in the second launch's epilogue.
#include "bgnn_internal.cuh"

namespace {

template <bool EXACT>
__device__ __forceinline__ float mac(float a, float b, float acc) {
  if constexpr (EXACT) {
    return __double2float_rn(__fma_rn((double)a, (double)b, (double)acc));
  } else {
    return __fmaf_rn(a, b, acc);
  }
}

// ---------------------------------------------------------------------------
// X*W: each output is one k-ascending chain owned by one thread (the
// reference's order), both operands moved by cp.async into a 4-stage
// shared-memory ring so no register staging or shared stores sit in the FMA
// stream.
//   A [m, k] row-major goes in transposed (As[k][m]) with 4-byte copies:
//     consecutive threads read consecutive k of one row (coalesced), and
//     the thread's 8 rows for one k come back as two 16-byte shared loads.
//   B [k, n] goes in as is, 16-byte copies when n % 4 == 0 (4-byte else).
//   Rows, columns and k beyond the matrix are zero-filled by the copy
//   (src-size 0) and never reach an output; the last partial k tile runs
//   only its real k steps (no fma with padding: it could turn -0 into +0).
// Tile 128 x BN (BN = 128: 8x8 per thread; BN = 64: 8x4), BK = 16.
// ---------------------------------------------------------------------------
constexpr int PG_BM = 128, PG_BK = 16, PG_S = 4, PG_APAD = 4;
constexpr int PG_UNROLL = 16;  // k steps per unrolled block: keeps the loop in the instruction cache

__device__ __forceinline__ void cpa4_zfill(float* s, const float* g, bool valid) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(s);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(g),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cpa16_zfill(float* s, const float* g, bool valid) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(s);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(g),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <int BN>
constexpr size_t pg_smem_bytes() {
  return (size_t)PG_S * (PG_BK * (PG_BM + PG_APAD) + PG_BK * BN) * sizeof(float);
}

// DUAL (the SAGE pair in one launch): the tile first runs A*B over k and
// stores it, rounded to f32, into its own outputs of C (the reference's
// St tensor); it then runs A2*B2 over k with that stored St as the addend,
// i.e. C = act(f32(f32(St + A2*B2) + bias)), bit for bit what two launches
// give, with one tile start-up and one launch instead of two.
template <int BN, bool EXACT, bool B16, bool V4OUT, bool DUAL = false>
__global__ void __launch_bounds__(256, 2) k_sgemm_pipe(const float* __restrict__ A,
                                                       const float* __restrict__ B, uint32_t m,
                                                       uint32_t k, uint32_t n,
                                                       const float* addend,
                                                       const float* __restrict__ bias, int act,
                                                       double act_param, float* C,
                                                       const float* __restrict__ A2,
                                                       const float* __restrict__ B2) {
  constexpr int TN = BN / 16;                 // 8 or 4 columns per thread
  constexpr int AST = PG_BM + PG_APAD;        // As row stride (floats)
  constexpr int A_STAGE = PG_BK * AST, B_STAGE = PG_BK * BN;
  extern __shared__ float4 pg_smem4[];
  float* smem = reinterpret_cast<float*>(pg_smem4);
  float* As = smem;                           // [S][BK][AST]
  float* Bs = smem + PG_S * A_STAGE;          // [S][BK][BN]
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const uint64_t m0 = (uint64_t)blockIdx.x * PG_BM;
  const uint32_t n0 = blockIdx.y * BN;
  const uint32_t nt1 = (k + PG_BK - 1) / PG_BK;  // k tiles per product
  const uint32_t ntiles = DUAL ? 2 * nt1 : nt1;

  // Per-thread copy pattern, fixed for every tile.  A: the thread copies
  // columns a_kk and a_kk + 8 of rows a_r + 32 j (j < 4); a warp covers 4
  // rows x 8 columns, 32-byte runs in global memory and 32 distinct banks in
  // the transposed tile (row stride = 4 mod 32).  B (16-byte): rows b_kk +
  // (256 / (BN/4)) i, columns b_c..b_c+3; B (4-byte): rows b_kk + (256 / BN) i,
  // column b_c.
  const int a_kk = tid % 8, a_r = tid / 8;
  const float* a_src = A + (m0 + a_r) * k + a_kk;
  float* a_dst = As + a_kk * AST + a_r;
  constexpr int B_COLS = B16 ? BN / 4 : BN;       // copies per B row
  constexpr int B_ROWS = 256 / B_COLS;            // B rows covered per pass
  constexpr int B_PASSES = PG_BK / B_ROWS;
  const int b_kk = tid / B_COLS, b_c = (tid % B_COLS) * (B16 ? 4 : 1);
  const bool b_col_ok = n0 + b_c < n;
  const float* b_src = B + (uint64_t)b_kk * n + n0 + b_c;
  float* b_dst = Bs + b_kk * BN + b_c;
  const float* a2_src = DUAL ? A2 + (m0 + a_r) * k + a_kk : nullptr;
  const float* b2_src = DUAL ? B2 + (uint64_t)b_kk * n + n0 + b_c : nullptr;

  auto load_stage = [&](uint32_t t, int slot) {
    const float* as_ = a_src;
    const float* bs_ = b_src;
    if constexpr (DUAL) {
      if (t >= nt1) {  // the second product
        t -= nt1;
        as_ = a2_src;
        bs_ = b2_src;
      }
    }
    const uint32_t k0 = t * PG_BK;
#pragma unroll
    for (int i = 0; i < (PG_BM * PG_BK) / 256; i++) {
      const int dk = 8 * (i % (PG_BK / 8)), dr = 32 * (i / (PG_BK / 8));
      const bool ok = k0 + a_kk + dk < k && m0 + a_r + dr < m;
      cpa4_zfill(a_dst + slot * A_STAGE + dk * AST + dr,
                 ok ? as_ + (uint64_t)dr * k + k0 + dk : A, ok);
    }
#pragma unroll
    for (int i = 0; i < B_PASSES; i++) {
      const uint32_t gk = k0 + b_kk + B_ROWS * i;
      const bool ok = b_col_ok && gk < k;
      const float* src = ok ? bs_ + (uint64_t)(k0 + B_ROWS * i) * n : B;
      float* dst = b_dst + slot * B_STAGE + B_ROWS * i * BN;
      if constexpr (B16)
        cpa16_zfill(dst, src, ok);
      else
        cpa4_zfill(dst, src, ok);
    }
  };

  // FAST: two adjacent columns share one packed fma.rn.f32x2 (two IEEE f32
  // fmas per instruction, each rounded exactly like fmaf), which halves the
  // FMA instructions the schedulers issue.  EXACT: the double-emulated step.
  // ROWPAIR (FAST, 4 columns per thread): the packed pairs run down two
  // adjacent rows instead, so the A pairs come straight from shared memory
  // and only the 4 B values are duplicated (4 moves per k step, not 8).
  constexpr int TP = TN / 2;
  constexpr bool ROWPAIR = !EXACT && TN == 4;
  float acc[8][TN];
  uint64_t accp[8][TP];  // FAST: (acc[i][2p], acc[i][2p+1]) packed
  uint64_t accr[4][4];   // ROWPAIR: (acc[2p][j], acc[2p+1][j]) packed
  auto zero = [&]() {
#pragma unroll
    for (int i = 0; i < 8; i++) {
#pragma unroll
      for (int j = 0; j < TN; j++) acc[i][j] = 0.0f;
#pragma unroll
      for (int q = 0; q < TP; q++) accp[i][q] = 0ull;
    }
#pragma unroll
    for (int p = 0; p < 4; p++)
#pragma unroll
      for (int j = 0; j < 4; j++) accr[p][j] = 0ull;
  };
  zero();
  // this thread's outputs (row i, columns 4h..4h+3) from whichever layout
  auto get4 = [&](int i, int h, float (&v)[4]) {
    if constexpr (EXACT) {
#pragma unroll
      for (int j = 0; j < 4; j++) v[j] = acc[i][h * 4 + j];
    } else if constexpr (ROWPAIR) {
#pragma unroll
      for (int j = 0; j < 4; j++) {
        float lo, hi;
        asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(accr[i >> 1][j]));
        v[j] = (i & 1) ? hi : lo;
      }
    } else {
      asm("mov.b64 {%0, %1}, %2;" : "=f"(v[0]), "=f"(v[1]) : "l"(accp[i][h * 2]));
      asm("mov.b64 {%0, %1}, %2;" : "=f"(v[2]), "=f"(v[3]) : "l"(accp[i][h * 2 + 1]));
    }
  };

  auto kstep = [&](const float* as, const float* bs, int kk) {
    if constexpr (ROWPAIR) {
      const ulonglong2 p0 = *reinterpret_cast<const ulonglong2*>(as + kk * AST + ty * 4);
      const ulonglong2 p1 = *reinterpret_cast<const ulonglong2*>(as + kk * AST + 64 + ty * 4);
      const uint64_t ap[4] = {p0.x, p0.y, p1.x, p1.y};
      const float4 b0 = *reinterpret_cast<const float4*>(bs + kk * BN + tx * 4);
      const float bw[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        uint64_t bd;
        asm("mov.b64 %0, {%1, %1};" : "=l"(bd) : "f"(bw[j]));
#pragma unroll
        for (int q = 0; q < 4; q++)
          asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(accr[q][j]) : "l"(ap[q]), "l"(bd), "l"(accr[q][j]));
      }
      return;
    }
    const float4 a0 = *reinterpret_cast<const float4*>(as + kk * AST + ty * 4);
    const float4 a1 = *reinterpret_cast<const float4*>(as + kk * AST + 64 + ty * 4);
    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    if constexpr (!EXACT) {
      uint64_t bp[TP];
      const ulonglong2 q0 = *reinterpret_cast<const ulonglong2*>(bs + kk * BN + tx * 4);
      bp[0] = q0.x;
      bp[1] = q0.y;
      if constexpr (TN == 8) {
        const ulonglong2 q1 = *reinterpret_cast<const ulonglong2*>(bs + kk * BN + 64 + tx * 4);
        bp[2] = q1.x;
        bp[3] = q1.y;
      }
#pragma unroll
      for (int i = 0; i < 8; i++) {
        uint64_t ad;
        asm("mov.b64 %0, {%1, %1};" : "=l"(ad) : "f"(av[i]));
#pragma unroll
        for (int q = 0; q < TP; q++)
          asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(accp[i][q]) : "l"(ad), "l"(bp[q]), "l"(accp[i][q]));
      }
      return;
    }
    float bv[TN];
    const float4 b0 = *reinterpret_cast<const float4*>(bs + kk * BN + tx * 4);
    bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
    if constexpr (TN == 8) {
      const float4 b1 = *reinterpret_cast<const float4*>(bs + kk * BN + 64 + tx * 4);
      bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
    }
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
      for (int j = 0; j < TN; j++) acc[i][j] = mac<EXACT>(av[i], bv[j], acc[i][j]);
  };

#pragma unroll
  for (int t = 0; t < PG_S - 1; t++) {
    if ((uint32_t)t < ntiles) load_stage(t, t);
    cpa_commit();
  }
  for (uint32_t t = 0; t < ntiles; t++) {
    cpa_wait<PG_S - 2>();  // this thread's copies of tile t have landed
    __syncthreads();       // ... everyone's; and tile t-1's slot is free
    const int slot = (int)(t % PG_S);
    const float* as = As + slot * A_STAGE;
    const float* bs = Bs + slot * B_STAGE;
    const uint32_t tk = (DUAL && t >= nt1) ? t - nt1 : t;      // k tile within its product
    const int kn = (int)min((uint32_t)PG_BK, k - tk * PG_BK);  // the last tile may be partial
    if (kn == PG_BK) {
      // the next stage's copies go out between the two halves of the tile,
      // so no warp issues them while the others wait at the barrier
#pragma unroll PG_UNROLL
      for (int kk = 0; kk < PG_BK / 2; kk++) kstep(as, bs, kk);
      if (t + PG_S - 1 < ntiles) load_stage(t + PG_S - 1, (int)((t + PG_S - 1) % PG_S));
      cpa_commit();
#pragma unroll PG_UNROLL
      for (int kk = PG_BK / 2; kk < PG_BK; kk++) kstep(as, bs, kk);
    } else {
      if (t + PG_S - 1 < ntiles) load_stage(t + PG_S - 1, (int)((t + PG_S - 1) % PG_S));
      cpa_commit();
      for (int kk = 0; kk < kn; kk++) kstep(as, bs, kk);
    }
    if constexpr (DUAL) {
      if (t == nt1 - 1) {
        // first product complete: store it as f32 into this thread's own
        // outputs (read back by this thread in the epilogue), restart
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const uint64_t gm = m0 + (i >> 2) * 64 + ty * 4 + (i & 3);
#pragma unroll
          for (int h = 0; h < TN / 4; h++) {
            const uint32_t gn = n0 + h * 64 + tx * 4;
            float v[4];
            get4(i, h, v);
            if (gm < m) {
              if (V4OUT && gn + 3 < n) {
                *reinterpret_cast<float4*>(C + gm * n + gn) = make_float4(v[0], v[1], v[2], v[3]);
              } else {
#pragma unroll
                for (int j = 0; j < 4; j++)
                  if (gn + j < n) C[gm * n + gn + j] = v[j];
              }
            }
          }
        }
        zero();
      }
    }
  }
  cpa_wait<0>();
  if constexpr (ROWPAIR) {
#pragma unroll
    for (int q = 0; q < 4; q++)
#pragma unroll
      for (int j = 0; j < 4; j++)
        asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[2 * q][j]), "=f"(acc[2 * q + 1][j]) : "l"(accr[q][j]));
  } else if constexpr (!EXACT) {
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
      for (int q = 0; q < TP; q++)
        asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[i][2 * q]), "=f"(acc[i][2 * q + 1]) : "l"(accp[i][q]));
  }

  // epilogue: f32(addend + acc), f32(+ bias), activation.  The addend may
  // be the output itself (the SAGE pair), so the compiler cannot move its
  // loads above earlier stores: each half of the thread's rows loads all of
  // its addend values first, then stores.
  float bv[TN];
#pragma unroll
  for (int h = 0; h < TN / 4; h++)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t gn = n0 + h * 64 + tx * 4 + j;
      bv[h * 4 + j] = (bias && gn < n) ? bias[gn] : 0.0f;
    }
#pragma unroll
  for (int half = 0; half < 2; half++) {
    float ad[4][TN];
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const uint64_t gm = m0 + half * 64 + ty * 4 + r;
#pragma unroll
      for (int h = 0; h < TN / 4; h++) {
        const uint32_t gn = n0 + h * 64 + tx * 4;
        if (addend && gm < m) {
          if (V4OUT && gn + 3 < n) {
            const float4 v = *reinterpret_cast<const float4*>(addend + gm * n + gn);
            ad[r][h * 4 + 0] = v.x; ad[r][h * 4 + 1] = v.y;
            ad[r][h * 4 + 2] = v.z; ad[r][h * 4 + 3] = v.w;
          } else {
#pragma unroll
            for (int j = 0; j < 4; j++) ad[r][h * 4 + j] = gn + j < n ? addend[gm * n + gn + j] : 0.0f;
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int i = half * 4 + r;
      const uint64_t gm = m0 + half * 64 + ty * 4 + r;
      if (gm >= m) continue;
#pragma unroll
      for (int h = 0; h < TN / 4; h++) {
        const uint32_t gn = n0 + h * 64 + tx * 4;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          float x = acc[i][h * 4 + j];
          if (addend) x = __fadd_rn(ad[r][h * 4 + j], x);
          if (bias) x = __fadd_rn(x, bv[h * 4 + j]);
          v[j] = apply_act(x, act, act_param);
        }
        if (V4OUT && gn + 3 < n) {
          *reinterpret_cast<float4*>(C + gm * n + gn) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; j++)
            if (gn + j < n) C[gm * n + gn + j] = v[j];
        }
      }
    }
  }
}

template <int BN, bool EXACT, bool B16, bool V4OUT, bool DUAL = false>
int launch_pipe_t(bgnn_ctx* ctx, const float* a, const float* b, uint32_t m, uint32_t k,
                  uint32_t n, const float* addend, const float* bias, int act, double act_param,
                  float* out, const float* a2 = nullptr, const float* b2 = nullptr) {
  constexpr size_t smem = pg_smem_bytes<BN>();
  auto kern = k_sgemm_pipe<BN, EXACT, B16, V4OUT, DUAL>;
  BGNN_CUDA(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
  dim3 grid((unsigned)((m + PG_BM - 1) / PG_BM), (n + BN - 1) / BN);
  kern<<<grid, 256, smem, ctx->stream>>>(a, b, m, k, n, addend, bias, act, act_param, out, a2,
                                         b2);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

// out = act(f32(f32(addend + a*b) + bias)), addend / bias optional.
// DUAL: out = act(f32(f32(f32(a*b) + a2*b2) + bias)) in one launch (addend
// must be out).
template <bool EXACT, bool DUAL = false>
int launch_pipe(bgnn_ctx* ctx, const float* a, const float* b, uint32_t m, uint32_t k,
                uint32_t n, const float* addend, const float* bias, int act, double act_param,
                float* out, const float* a2 = nullptr, const float* b2 = nullptr) {
  const bool b16 = (n % 4 == 0) && ((uintptr_t)b % 16 == 0) && ((uintptr_t)b2 % 16 == 0);
  const bool v4 = (n % 4 == 0) && ((uintptr_t)out % 16 == 0) &&
                  (addend == nullptr || (uintptr_t)addend % 16 == 0);
  if (n <= 64) {
    if (b16)
      return v4 ? launch_pipe_t<64, EXACT, true, true, DUAL>(
                      ctx, a, b, m, k, n, addend, bias, act, act_param, out, a2, b2)
                : launch_pipe_t<64, EXACT, true, false, DUAL>(
                      ctx, a, b, m, k, n, addend, bias, act, act_param, out, a2, b2);
    return launch_pipe_t<64, EXACT, false, false, DUAL>(
        ctx, a, b, m, k, n, addend, bias, act, act_param, out, a2, b2);
  }
  if (b16)
    return v4 ? launch_pipe_t<128, EXACT, true, true, DUAL>(
                    ctx, a, b, m, k, n, addend, bias, act, act_param, out, a2, b2)
              : launch_pipe_t<128, EXACT, true, false, DUAL>(
                    ctx, a, b, m, k, n, addend, bias, act, act_param, out, a2, b2);
  return launch_pipe_t<128, EXACT, false, false, DUAL>(
      ctx, a, b, m, k, n, addend, bias, act, act_param, out, a2, b2);
}

}  // namespace

namespace {

// ---- elementwise -----------------------------------------------------------
__global__ void k_act(int act, double p, const float* __restrict__ x, uint64_t n,
                      float* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = apply_act(x[i], act, p);
}

__global__ void k_add(const float* __restrict__ a, const float* __restrict__ b, uint64_t n,
                      float* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = __fadd_rn(a[i], b[i]);
}

// SAGE L2 normalise (sage.ts:199-214): norm = sqrt(sum v*v) in double,
// sequential over the row; out = f32(v / norm) when norm > 0.
__global__ void k_l2norm(float* x, uint32_t m, uint32_t n) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < m; r += gridDim.x * blockDim.x) {
    float* row = x + (uint64_t)r * n;
    double s = 0.0;
    for (uint32_t f = 0; f < n; f++) {
      const double v = (double)row[f];
      s = __dadd_rn(s, __dmul_rn(v, v));
    }
    const double nrm = __dsqrt_rn(s);
    if (nrm > 0.0)
      for (uint32_t f = 0; f < n; f++) row[f] = __double2float_rn(__ddiv_rn((double)row[f], nrm));
  }
}

__global__ void k_gather_rows(const float* __restrict__ x, uint32_t nx,
                              const uint32_t* __restrict__ idx, uint64_t n, uint32_t f,
                              float* __restrict__ out, int* err) {
  const uint64_t total = n * f;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = t / f;
    const uint32_t c = (uint32_t)(t - i * f);
    const uint32_t s = idx[i];
    if (s >= nx) {
      if (c == 0) dev_raise(err, DEVERR_INDEX, i, 1);
      out[t] = 0.0f;
    } else {
      out[t] = x[(uint64_t)s * f + c];
    }
  }
}

// wasmSpmv (index.ts:304-335): double accumulator, one rounding at the store
__global__ void k_spmv(const uint32_t* __restrict__ rp, const uint32_t* __restrict__ col,
                       const float* __restrict__ val, const float* __restrict__ x, uint32_t rows,
                       float* __restrict__ out) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    double s = 0.0;
    for (uint32_t j = rp[r]; j < rp[r + 1]; j++)
      s = __dadd_rn(s, __dmul_rn((double)val[j], (double)x[col[j]]));
    out[r] = __double2float_rn(s);
  }
}

// SAGE pool projection (sage.ts:149-159): sum = bias[j] + sum_k x*w with a
// double accumulator (no per-step f32 store), stored as f32(Math.max(0, sum)).
__global__ void k_pool_proj(const float* __restrict__ x, const float* __restrict__ w,
                            const float* __restrict__ b, uint32_t m, uint32_t k,
                            float* __restrict__ out) {
  const uint64_t total = (uint64_t)m * k;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = t / k;
    const uint32_t j = (uint32_t)(t - i * k);
    double s = b ? (double)b[j] : 0.0;
    const float* xr = x + i * k;
    for (uint32_t q = 0; q < k; q++) s = __dadd_rn(s, __dmul_rn((double)xr[q], (double)w[(uint64_t)q * k + j]));
    out[t] = (s != s) ? __double2float_rn(s) : (s > 0.0 ? __double2float_rn(s) : 0.0f);
  }
}

inline unsigned grid_for(bgnn_ctx* ctx, uint64_t n, int tpb) {
  uint64_t b = (n + tpb - 1) / tpb;
  const uint64_t cap = (uint64_t)ctx->num_sms * 16;
  if (b > cap) b = cap;
  if (b == 0) b = 1;
  return (unsigned)b;
}

}  // namespace

int bgnn_run_linear(bgnn_ctx* ctx, const float* a, const float* w, const float* a2,
                    const float* w2, uint32_t m, uint32_t k, uint32_t n, const float* bias,
                    int act, double act_param, float* out) {
  if (m == 0 || n == 0) return BGNN_OK;
  // k == 0 runs no mac step: the output is act(0 + bias), as in the reference
  const bool dual = a2 != nullptr && w2 != nullptr;
  const bool exact = ctx->math == BGNN_MATH_EXACT;
  if (ctx->math == BGNN_MATH_TENSOR && k > 0) {
    const int rc = bgnn_run_linear_tc(ctx, a, w, k, dual ? a2 : nullptr, dual ? w2 : nullptr,
                                      dual ? k : 0, m, n, nullptr, bias, act, act_param, out);
    if (rc != BGNN_ERR_UNSUPPORTED) return rc;
  }
  // SAGE pair: St = a2*w2 stored as f32 (the reference's Tensor), then
  // f32(St + a*w) (+ bias, activation); one launch runs both products per
  // output tile (k == 0 keeps two launches: the first writes St = 0)
  if (dual && k > 0)
    return exact ? launch_pipe<true, true>(ctx, a2, w2, m, k, n, out, bias, act, act_param, out,
                                           a, w)
                 : launch_pipe<false, true>(ctx, a2, w2, m, k, n, out, bias, act, act_param, out,
                                            a, w);
  if (dual) {
    BGNN_TRY(exact ? launch_pipe<true>(ctx, a2, w2, m, k, n, nullptr, nullptr, 0, 0.0, out)
                   : launch_pipe<false>(ctx, a2, w2, m, k, n, nullptr, nullptr, 0, 0.0, out));
  }
  const float* addend = dual ? out : nullptr;
  return exact ? launch_pipe<true>(ctx, a, w, m, k, n, addend, bias, act, act_param, out)
               : launch_pipe<false>(ctx, a, w, m, k, n, addend, bias, act, act_param, out);
}

int bgnn_run_linear_add(bgnn_ctx* ctx, const float* a, const float* w, uint32_t m, uint32_t k,
                        uint32_t n, const float* addend, const float* bias, int act,
                        double act_param, float* out) {
  if (m == 0 || n == 0) return BGNN_OK;
  if (ctx->math == BGNN_MATH_TENSOR && k > 0) {
    const int rc = bgnn_run_linear_tc(ctx, a, w, k, nullptr, nullptr, 0, m, n, addend, bias, act,
                                      act_param, out);
    if (rc != BGNN_ERR_UNSUPPORTED) return rc;
  }
  return ctx->math == BGNN_MATH_EXACT
             ? launch_pipe<true>(ctx, a, w, m, k, n, addend, bias, act, act_param, out)
             : launch_pipe<false>(ctx, a, w, m, k, n, addend, bias, act, act_param, out);
}

int bgnn_run_activation(bgnn_ctx* ctx, int act, double param, const float* x, uint64_t n,
                        float* out) {
  if (n == 0) return BGNN_OK;
  k_act<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(act, param, x, n, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_run_add(bgnn_ctx* ctx, const float* a, const float* b, uint64_t n, float* out) {
  if (n == 0) return BGNN_OK;
  k_add<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(a, b, n, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_run_l2norm(bgnn_ctx* ctx, float* x, uint32_t m, uint32_t n) {
  if (m == 0 || n == 0) return BGNN_OK;
  k_l2norm<<<grid_for(ctx, m, 128), 128, 0, ctx->stream>>>(x, m, n);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_run_gather_rows(bgnn_ctx* ctx, const float* x, uint32_t nx, const uint32_t* idx,
                         uint64_t n, uint32_t f, float* out) {
  if (n == 0 || f == 0) return BGNN_OK;
  k_gather_rows<<<grid_for(ctx, n * f, 256), 256, 0, ctx->stream>>>(x, nx, idx, n, f, out,
                                                                      ctx->d_err);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_run_spmv(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col, const float* val,
                  const float* x, uint32_t num_rows, float* out) {
  if (num_rows == 0) return BGNN_OK;
  k_spmv<<<grid_for(ctx, num_rows, 128), 128, 0, ctx->stream>>>(row_ptr, col, val, x, num_rows, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

extern "C" int bgnn_pool_projection(bgnn_ctx* ctx, const float* x, const float* w,
                                    const float* bias, uint32_t m, uint32_t k, float* out) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, (x && w && out) || (uint64_t)m * k == 0, "NULL argument");
  if ((uint64_t)m * k == 0) return BGNN_OK;
  k_pool_proj<<<grid_for(ctx, (uint64_t)m * k, 256), 256, 0, ctx->stream>>>(x, w, bias, m, k, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}
