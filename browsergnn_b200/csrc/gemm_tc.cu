// X*W on the 5th-generation tensor cores (tcgen05.mma kind::tf32) with a
// 3xTF32 split: a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi, where x_hi is x
// rounded to TF32 (cvt.rna.tf32.f32) and x_lo = x - x_hi (exact in f32).  The
// three products accumulate in f32 in tensor memory, which gives f32-level
// accuracy -- but not the reference's summation order: wasmMatmul
// (src/backend/wasm/index.ts:18-63) rounds to f32 after every k step in
// ascending k, and no tensor-core order reproduces those roundings.  This
// path therefore runs only in the BGNN_MATH_TENSOR mode; the default keeps
// X*W on the FP32 pipe in the reference's order (gemm.cu).
//
// Accumulation: the tensor core adds its products into the f32 accumulator
// with its own rounding, and over a whole K that error reaches the size of
// the 1e-5 relative bar (measured: 3.9% of a SAGE layer's elements outside
// it).  So each 32-wide k block goes into its own tensor-memory buffer (four
// in rotation) and the epilogue warps add the block's partial sums into f32
// registers with round-to-nearest ("promotion"): the tensor core then only
// ever sums 12 products.
//
// Schedule: a persistent kernel, one CTA per SM, 128-row output tiles of
// NT columns (NT = the output width rounded up to 16, at most 128: the
// epilogue holds a row's NT sums in registers).  Warp roles:
//   warp 8     TMA producer: per 32-wide k block, the A rows (128 x 32 f32,
//              128-byte swizzle) and the pre-split B_hi / B_lo tiles
//              (NT x 32, K-major) into a ring of shared-memory stages;
//   warps 4-7  splitter: rewrites the A tile as A_hi in place and writes
//              A_lo beside it (same offsets, so the swizzle carries over),
//              then fences the generic-proxy writes for the tensor core;
//   warp 9     MMA issuer (one thread): 3 x 4 tcgen05.mma (M=128, N=NT,
//              K=8) per k block into the block's tensor-memory buffer; one
//              tcgen05.commit frees the stage, another marks the buffer full;
//   warps 0-3  epilogue: per k block, tcgen05.ld of its 32 lanes (rows) of
//              the buffer and f32 adds into registers; after the last block
//              f32(addend + sum), + bias, activation, stores.
// Every mbarrier wait is bounded; a wait that gives up raises the context's
// error word (BGNN_ERR_TIMEOUT at the next synchronisation), tells the other
// roles through shared memory and the CTA frees its tensor memory and exits.
// Two operand segments (A1*B1 + A2*B2, the SAGE pair) accumulate into the
// same tile.  TMA loads never use multicast and read only this GPU's memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "bgnn_internal.cuh"

namespace {

constexpr int TC_BM = 128;
constexpr int TC_BK = 32;                     // f32 per k block: one 128-byte swizzle row
constexpr int TC_THREADS = 320;               // 10 warps
constexpr uint32_t TC_SPIN_LIMIT = 1u << 24;  // try_wait polls before a wait gives up

constexpr int TC_BUFS = 4;  // k-block accumulators in tensor memory

template <int NT>
struct TcCfg {
  static_assert(NT % 16 == 0 && NT <= 128, "tile width");
  static constexpr int STAGES = NT >= 128 ? 3 : 4;
  static constexpr int A_BYTES = TC_BM * TC_BK * 4;  // 16 KB
  static constexpr int B_BYTES = NT * TC_BK * 4;
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int TMEM_COLS = TC_BUFS * NT <= 32 ? 32 : TC_BUFS * NT <= 64 ? 64
                                 : TC_BUFS * NT <= 128 ? 128 : TC_BUFS * NT <= 256 ? 256 : 512;
  static constexpr uint32_t TX = A_BYTES + 2 * B_BYTES;  // bytes the TMA brings per stage
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
  static_assert(B_BYTES % 1024 == 0, "every operand tile starts on a 1024-byte swizzle atom");
  static_assert(SMEM <= 227 * 1024, "stages fit in shared memory");
  // instruction descriptor: D f32, A/B tf32, both K-major, N = NT, M = 128
  static constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) |
                                    ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
};

struct TcArgs {
  uint32_t m, n, k1, k2;  // k2 == 0: one operand segment
  const float* addend;
  const float* bias;
  int act;
  double act_param;
  float* out;
  int* err;
};

__device__ __forceinline__ uint32_t s_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait; false when it gave up or another role already did
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, volatile uint32_t* abort_flag,
                                          int* err, int where) {
  for (uint32_t i = 0; i < TC_SPIN_LIMIT; i++) {
    if (mbar_try(a, parity)) return true;
    if (*abort_flag) return false;
  }
  *abort_flag = 1u;
  dev_raise(err, DEVERR_TIMEOUT, (uint64_t)blockIdx.x, where);
  return false;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 bytes apart (stride byte offset), version 1 (Blackwell)
__device__ __forceinline__ uint64_t smem_desc(uint32_t a) {
  return (uint64_t)((a & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 16; j++) v[j] = __uint_as_float(r[j]);
}

template <int NT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap ta1, const __grid_constant__ CUtensorMap tbh1,
              const __grid_constant__ CUtensorMap tbl1, const __grid_constant__ CUtensorMap ta2,
              const __grid_constant__ CUtensorMap tbh2, const __grid_constant__ CUtensorMap tbl2,
              const TcArgs a) {
  using C = TcCfg<NT>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t tc_smem[];
  const uint32_t raw = s_addr(tc_smem);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzle atoms start on 1024 bytes
  uint8_t* gbase = tc_smem + (base - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + (size_t)S * C::STAGE_BYTES);
  // full[S] (TMA landed), split[S] (A split), empty[S] (MMAs done with the
  // stage), accf[B] (k-block partials ready), acce[B] (partials drained)
  const uint32_t b_full = s_addr(bars), b_split = b_full + 8 * S, b_empty = b_split + 8 * S;
  const uint32_t b_accf = b_empty + 8 * S, b_acce = b_accf + 8 * TC_BUFS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 2 * TC_BUFS);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(b_full + 8 * s, 1);
      mbar_init(b_split + 8 * s, 128);
      mbar_init(b_empty + 8 * s, 1);
    }
    for (int b = 0; b < TC_BUFS; b++) {
      mbar_init(b_accf + 8 * b, 1);
      mbar_init(b_acce + 8 * b, 128);
    }
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     s_addr(tmem_slot)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const uint32_t m_tiles = (a.m + TC_BM - 1) / TC_BM, n_tiles = (a.n + NT - 1) / NT;
  const uint32_t tiles = m_tiles * n_tiles;
  const uint32_t nkb1 = (a.k1 + TC_BK - 1) / TC_BK, nkb2 = (a.k2 + TC_BK - 1) / TC_BK;
  const uint32_t nkb = nkb1 + nkb2;
  auto stage_addr = [&](int s) { return base + (uint32_t)s * C::STAGE_BYTES; };

  if (warp == 8) {
    // ---- TMA producer ----
    if (lane == 0 && nkb > 0) {
      int s = 0;
      uint32_t ph = 0;
      for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int m0 = (int)((t / n_tiles) * TC_BM), n0 = (int)((t % n_tiles) * NT);
        for (uint32_t kb = 0; kb < nkb; kb++) {
          if (!mbar_wait(b_empty + 8 * s, ph ^ 1u, abort_flag, a.err, 50)) goto done;
          mbar_expect_tx(b_full + 8 * s, C::TX);
          const bool seg2 = kb >= nkb1;
          const int kx = (int)((seg2 ? kb - nkb1 : kb) * TC_BK);
          const uint32_t st = stage_addr(s);
          tma_load_2d(st, seg2 ? &ta2 : &ta1, kx, m0, b_full + 8 * s);
          tma_load_2d(st + 2 * C::A_BYTES, seg2 ? &tbh2 : &tbh1, kx, n0, b_full + 8 * s);
          tma_load_2d(st + 2 * C::A_BYTES + C::B_BYTES, seg2 ? &tbl2 : &tbl1, kx, n0,
                      b_full + 8 * s);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 9) {
    // ---- MMA issuer ----
    if (lane == 0 && nkb > 0) {
      int s = 0, buf = 0;
      uint32_t ph = 0, aph = 0;
      for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        for (uint32_t kb = 0; kb < nkb; kb++) {
          if (!mbar_wait(b_acce + 8 * buf, aph ^ 1u, abort_flag, a.err, 51)) goto done;
          if (!mbar_wait(b_split + 8 * s, ph, abort_flag, a.err, 52)) goto done;
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(buf * NT);
          const uint32_t st = stage_addr(s);
#pragma unroll
          for (int kk = 0; kk < TC_BK / 8; kk++) {
            const uint32_t off = (uint32_t)kk * 32u;  // 8 tf32 = 32 bytes along the row
            const uint64_t ah = smem_desc(st + off), al = smem_desc(st + C::A_BYTES + off);
            const uint64_t bh = smem_desc(st + 2 * C::A_BYTES + off);
            const uint64_t bl = smem_desc(st + 2 * C::A_BYTES + C::B_BYTES + off);
            // small terms first; the block's first product starts the buffer
            mma_tf32(d, al, bh, C::IDESC, kk != 0 ? 1u : 0u);
            mma_tf32(d, ah, bl, C::IDESC, 1u);
            mma_tf32(d, ah, bh, C::IDESC, 1u);
          }
          mma_commit(b_empty + 8 * s);
          mma_commit(b_accf + 8 * buf);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
          if (++buf == TC_BUFS) {
            buf = 0;
            aph ^= 1u;
          }
        }
      }
    }
  } else if (warp >= 4) {
    // ---- splitter: A -> A_hi (in place) + A_lo ----
    const int tid = threadIdx.x - 128;
    int s = 0;
    uint32_t ph = 0;
    for (uint32_t t = blockIdx.x; t < tiles && nkb > 0; t += gridDim.x) {
      for (uint32_t kb = 0; kb < nkb; kb++) {
        if (!mbar_wait(b_full + 8 * s, ph, abort_flag, a.err, 53)) goto done;
        float4* ah = reinterpret_cast<float4*>(gbase + (size_t)s * C::STAGE_BYTES);
        float4* al = reinterpret_cast<float4*>(gbase + (size_t)s * C::STAGE_BYTES + C::A_BYTES);
#pragma unroll
        for (int i = 0; i < C::A_BYTES / 16 / 128; i++) {
          const int q = tid + i * 128;
          const float4 v = ah[q];
          float4 h, l;
          h.x = __uint_as_float(to_tf32(v.x));
          h.y = __uint_as_float(to_tf32(v.y));
          h.z = __uint_as_float(to_tf32(v.z));
          h.w = __uint_as_float(to_tf32(v.w));
          l.x = __fsub_rn(v.x, h.x);
          l.y = __fsub_rn(v.y, h.y);
          l.z = __fsub_rn(v.z, h.z);
          l.w = __fsub_rn(v.w, h.w);
          ah[q] = h;
          al[q] = l;
        }
        // make these generic-proxy writes visible to the tensor core
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(b_split + 8 * s);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else {
    // ---- epilogue: warp w reads accumulator lanes (rows) 32w .. 32w+31 ----
    int buf = 0;
    uint32_t aph = 0;
    const bool v4 = (a.n % 4u) == 0u;
    for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x) {
      const uint32_t m0 = (t / n_tiles) * TC_BM, n0 = (t % n_tiles) * NT;
      const uint32_t row = m0 + (uint32_t)threadIdx.x;
      float acc[NT];
#pragma unroll
      for (int j = 0; j < NT; j++) acc[j] = 0.0f;
      for (uint32_t kb = 0; kb < nkb; kb++) {
        if (!mbar_wait(b_accf + 8 * buf, aph, abort_flag, a.err, 54)) goto done;
        tc_fence_after();
        const uint32_t tb = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * NT);
#pragma unroll
        for (int c = 0; c < NT / 16; c++) {
          float v[16];
          tmem_ld16(tb + (uint32_t)(c * 16), v);
#pragma unroll
          for (int j = 0; j < 16; j++) acc[c * 16 + j] = __fadd_rn(acc[c * 16 + j], v[j]);
        }
        tc_fence_before();
        mbar_arrive(b_acce + 8 * buf);
        if (++buf == TC_BUFS) {
          buf = 0;
          aph ^= 1u;
        }
      }
      if (row >= a.m) continue;
      float* orow = a.out + (uint64_t)row * a.n;
      const float* arow = a.addend ? a.addend + (uint64_t)row * a.n : nullptr;
#pragma unroll
      for (int c = 0; c < NT / 4; c++) {
        const uint32_t col = n0 + (uint32_t)c * 4u;
        if (col >= a.n) break;
        float x[4] = {acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]};
        if (v4) {
          if (arow) {
            const float4 y = *reinterpret_cast<const float4*>(arow + col);
            x[0] = __fadd_rn(y.x, x[0]);
            x[1] = __fadd_rn(y.y, x[1]);
            x[2] = __fadd_rn(y.z, x[2]);
            x[3] = __fadd_rn(y.w, x[3]);
          }
#pragma unroll
          for (int j = 0; j < 4; j++) {
            if (a.bias) x[j] = __fadd_rn(x[j], a.bias[col + j]);
            x[j] = apply_act(x[j], a.act, a.act_param);
          }
          *reinterpret_cast<float4*>(orow + col) = make_float4(x[0], x[1], x[2], x[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            if (col + (uint32_t)j < a.n) {
              float y = x[j];
              if (arow) y = __fadd_rn(arow[col + j], y);
              if (a.bias) y = __fadd_rn(y, a.bias[col + j]);
              orow[col + j] = apply_act(y, a.act, a.act_param);
            }
          }
        }
      }
    }
  }
done:
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::TMEM_COLS)
                 : "memory");
  }
}

// B [k, n] row-major -> Bt_hi, Bt_lo [n, k] (K-major, as the MMA reads B)
__global__ void k_split_bt(const float* __restrict__ w, uint32_t k, uint32_t n,
                           float* __restrict__ hi, float* __restrict__ lo) {
  const uint64_t total = (uint64_t)k * n;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = (uint32_t)(t / k), q = (uint32_t)(t - (uint64_t)j * k);
    const float x = w[(uint64_t)q * n + j];
    const float h = __uint_as_float(to_tf32(x));
    hi[t] = h;
    lo[t] = __fsub_rn(x, h);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn(bgnn_ctx* ctx) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  (void)ctx;
  return fn;
}

// [rows, inner] f32 row-major, boxes of 32 x box_rows, 128-byte swizzle,
// out-of-range elements read as zero
int make_map(bgnn_ctx* ctx, CUtensorMap* map, const float* base, uint64_t inner, uint64_t rows,
             uint32_t box_rows) {
  auto enc = encode_fn(ctx);
  if (!enc) return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 4};
  cuuint32_t box[2] = {(cuuint32_t)TC_BK, box_rows};
  cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                         strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "tensor map encode failed (%d)", (int)r);
  return BGNN_OK;
}

template <int NT>
int launch_tc(bgnn_ctx* ctx, const CUtensorMap* maps, const TcArgs& args) {
  using C = TcCfg<NT>;
  BGNN_CUDA(ctx, cudaFuncSetAttribute(k_gemm_tc<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)C::SMEM));
  const uint64_t tiles = ((uint64_t)(args.m + TC_BM - 1) / TC_BM) * ((args.n + NT - 1) / NT);
  const int sms = ctx->grid_sms > 0 && ctx->grid_sms < ctx->num_sms ? ctx->grid_sms : ctx->num_sms;
  const unsigned grid = (unsigned)(tiles < (uint64_t)sms ? (tiles ? tiles : 1) : sms);
  k_gemm_tc<NT><<<grid, TC_THREADS, C::SMEM, ctx->stream>>>(maps[0], maps[1], maps[2], maps[3],
                                                             maps[4], maps[5], args);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

}  // namespace

int bgnn_run_linear_tc(bgnn_ctx* ctx, const float* a1, const float* w1, uint32_t k1,
                       const float* a2, const float* w2, uint32_t k2, uint32_t m, uint32_t n,
                       const float* addend, const float* bias, int act, double act_param,
                       float* out) {
  if (m == 0 || n == 0) return BGNN_OK;
  // TMA: 16-byte aligned bases and row strides (k % 4 == 0)
  auto ok_ptr = [](const void* p) { return ((uintptr_t)p & 15u) == 0; };
  if (k1 % 4 || k2 % 4 || !ok_ptr(a1) || (k2 && !ok_ptr(a2)) || (k1 + k2 == 0))
    return BGNN_ERR_UNSUPPORTED;
  // tile width: the output width rounded up to 16 (wider outputs take
  // several 128-column tiles)
  const int nt = n <= 32 ? 32 : n <= 48 ? 48 : n <= 64 ? 64 : n <= 96 ? 96 : 128;
  // B operands split once per call: [n, k] hi and lo per segment
  DevTmp bsplit;
  const uint64_t b1 = (uint64_t)n * k1, b2 = (uint64_t)n * k2;
  BGNN_TRY(bgnn_tmp_alloc(ctx, bsplit, (2 * b1 + 2 * b2 + 8) * sizeof(float)));
  float* bh1 = bsplit.as<float>();
  float* bl1 = bh1 + b1;
  float* bh2 = bl1 + b1;
  float* bl2 = bh2 + b2;
  // keep every operand base 16-byte aligned
  if (((uintptr_t)bh2 & 15u) || ((uintptr_t)bl1 & 15u)) return BGNN_ERR_UNSUPPORTED;
  auto split = [&](const float* w, uint32_t k, float* hi, float* lo) -> int {
    const uint64_t tot = (uint64_t)k * n;
    uint64_t blocks = (tot + 255) / 256;
    if (blocks > (uint64_t)ctx->num_sms * 8) blocks = (uint64_t)ctx->num_sms * 8;
    k_split_bt<<<(unsigned)(blocks ? blocks : 1), 256, 0, ctx->stream>>>(w, k, n, hi, lo);
    BGNN_LAUNCHED(ctx);
    return BGNN_OK;
  };
  if (k1) BGNN_TRY(split(w1, k1, bh1, bl1));
  if (k2) BGNN_TRY(split(w2, k2, bh2, bl2));
  CUtensorMap maps[6];
  const uint32_t nbox = (uint32_t)nt;
  // an empty first segment still needs well-formed maps: reuse the second's
  const float* ma = k1 ? a1 : a2;
  const uint32_t mk = k1 ? k1 : k2;
  BGNN_TRY(make_map(ctx, &maps[0], ma, mk, m, TC_BM));
  BGNN_TRY(make_map(ctx, &maps[1], k1 ? bh1 : bh2, mk, n, nbox));
  BGNN_TRY(make_map(ctx, &maps[2], k1 ? bl1 : bl2, mk, n, nbox));
  if (k2) {
    BGNN_TRY(make_map(ctx, &maps[3], a2, k2, m, TC_BM));
    BGNN_TRY(make_map(ctx, &maps[4], bh2, k2, n, nbox));
    BGNN_TRY(make_map(ctx, &maps[5], bl2, k2, n, nbox));
  } else {
    maps[3] = maps[0];
    maps[4] = maps[1];
    maps[5] = maps[2];
  }
  TcArgs args;
  args.m = m;
  args.n = n;
  args.k1 = k1 ? k1 : k2;
  args.k2 = k1 ? k2 : 0;
  args.addend = addend;
  args.bias = bias;
  args.act = act;
  args.act_param = act_param;
  args.out = out;
  args.err = ctx->d_err;
  switch (nt) {
    case 32: return launch_tc<32>(ctx, maps, args);
    case 48: return launch_tc<48>(ctx, maps, args);
    case 64: return launch_tc<64>(ctx, maps, args);
    case 96: return launch_tc<96>(ctx, maps, args);
    default: return launch_tc<128>(ctx, maps, args);
  }
}
