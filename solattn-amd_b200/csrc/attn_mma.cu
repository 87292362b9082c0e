// Fused routed attention, 64-row q-block per CTA, mma.sync BF16 tiles.
// (Replaces `_sol`, kernels.py:101-182.)  Runs only for more than 4096 key blocks
// (T > 262144 keys); every other launch takes the tcgen05 kernel of attn_sm100.cu.
//
// CTA = 4 warps, one (b, h, q-block); warp w owns rows 16w..16w+15.
//   1. Prologue: Q tile -> shared (cp.async, zero-filled past Tq); routing of every key block
//      (one warp ballot per 32 blocks, rule in common.cuh:route_selected) into a shared
//      bitmask; warp 0 compacts it into a tile list: first every 64-centroid tile that holds
//      at least one unselected block, then every selected key block in increasing order.
//   2. Main loop over the tile list with double-buffered K/V tiles (cp.async): S = Q K^T
//      (mma.m16n8k16), log2-domain scaling plus a per-column bias (0 / -inf for exact tiles,
//      log2(len) / -inf for centroid tiles, -inf where the centroid's block is exact), one
//      FP32 online softmax (max, denominator) per row, BF16 P, O += P V.
//   3. Epilogue: O / l -> BF16, staged through shared memory, 16-byte coalesced stores into the
//      contiguous [B, Tq, H, D] output; counts[b, qb, h] = number of exact blocks.
#include "common.cuh"

namespace solattn {

namespace {

template <int D>
struct MmaSmem {
  static constexpr int kTile = kBlock * D;  // elements of one 64 x D tile
  static size_t bytes(int nkb) {
    const int nwords = (nkb + 31) / 32;
    const int nct = (nkb + 63) / 64;
    return (size_t)5 * kTile * 2 + 2 * kBlock * 4 + D * 4 + (size_t)nwords * 4 +
           (size_t)(nct + nkb) * 4 + 16;
  }
};

__device__ __forceinline__ uint32_t valid_bits(int w, int nkb) {
  const int lo = 32 * w;
  if (lo + 32 <= nkb) return 0xffffffffu;
  if (lo >= nkb) return 0u;
  return (1u << (nkb - lo)) - 1u;
}

}  // namespace

template <int D>
__global__ void __launch_bounds__(128) attn_mma_kernel(const AttnParams p) {
  constexpr int kTile = MmaSmem<D>::kTile;
  constexpr int kChunks = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sK = sQ + kTile;      // [2][kTile]
  __nv_bfloat16* sV = sK + 2 * kTile;  // [2][kTile]
  float* sBias = reinterpret_cast<float*>(sV + 2 * kTile);  // [2][64]
  float* sQbar = sBias + 2 * kBlock;                          // [D]
  uint32_t* sMask = reinterpret_cast<uint32_t*>(sQbar + D);
  const int nwords = (p.nkb + 31) / 32;
  int* sTiles = reinterpret_cast<int*>(sMask + nwords);
  __shared__ int sNum, sNsel;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qb = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int q0 = qb * kBlock;
  // The batch's keys: its own count in a ragged launch (rows past it are never read).
  const int tk = key_count(p, b), nkb_b = (tk + kBlock - 1) / kBlock;

  // ---- Q tile (cp.async, zero-fill past Tq) ----
  {
    const uint32_t base = smem_u32(sQ);
    const int chunk = tid % kChunks;
    for (int r = tid / kChunks; r < kBlock; r += 128 / kChunks) {
      const bool ok = q0 + r < p.Tq;
      const __nv_bfloat16* src = ok ? row_ptr(p.q, p.Tq, b, h, q0 + r, p.status) : p.q.ptr;
      cp_async16(swz<D>(base, r, chunk), src + (ok ? chunk * 8 : 0), ok ? 16 : 0);
    }
    cp_async_commit();
  }
  float cut = 0.f;
  if (p.force == 0) {
    for (int d = tid; d < D; d += 128) sQbar[d] = p.qc[((int64_t)bh * p.nqb + qb) * D + d];
    cut = p.cutoff[(int64_t)bh * p.nqb + qb];
  }
  __syncthreads();

  // ---- routing bitmask ----
  const __nv_bfloat16* kc_bh = p.kc + (int64_t)bh * p.nkb * D;
  for (int w = warp; w < nwords; w += 4) {
    const int kb = 32 * w + lane;
    const bool sel = kb < nkb_b && route_selected(p, sQbar, kc_bh + (int64_t)kb * D, cut, D, b, qb, kb);
    const uint32_t bal = __ballot_sync(0xffffffffu, sel);
    if (lane == 0) {
      sMask[w] = bal;
      if (p.masks) p.masks[((int64_t)bh * p.nqb + qb) * nwords + w] = bal;
    }
  }
  __syncthreads();

  // ---- tile list (warp 0) ----
  if (warp == 0) {
    int base = 0;
    const int nct = (nkb_b + 63) / 64;
    if (p.force != 1) {
      for (int t0 = 0; t0 < nct; t0 += 32) {
        const int t = t0 + lane;
        bool want = false;
        if (t < nct) {
          const uint32_t w0 = sMask[2 * t];
          const uint32_t w1 = (2 * t + 1 < nwords) ? sMask[2 * t + 1] : 0xffffffffu;
          want = ((~w0 & valid_bits(2 * t, nkb_b)) | (~w1 & valid_bits(2 * t + 1, nkb_b))) != 0u;
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, want);
        if (want) sTiles[base + __popc(bal & ((1u << lane) - 1u))] = -(t + 1);
        base += __popc(bal);
      }
    }
    const int exact0 = base;
    for (int w0 = 0; w0 < nwords; w0 += 32) {
      const int w = w0 + lane;
      uint32_t bits = (w < nwords) ? sMask[w] : 0u;
      const int cnt = __popc(bits);
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int off = base + incl - cnt;
      while (bits) {
        const int bit = __ffs(bits) - 1;
        sTiles[off++] = 32 * w + bit;
        bits &= bits - 1u;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      sNum = base;
      sNsel = base - exact0;
    }
  }
  __syncthreads();
  const int ntiles = sNum;
  if (p.counts && tid == 0) p.counts[((int64_t)b * p.nqb + qb) * p.H + h] = sNsel;

  // ---- tile loader ----
  const __nv_bfloat16* vc_bh = p.vc + (int64_t)bh * p.nkb * D;
  auto load_tile = [&](int i, int buf) {
    const int e = sTiles[i];
    const uint32_t kbase = smem_u32(sK + buf * kTile);
    const uint32_t vbase = smem_u32(sV + buf * kTile);
    const int chunk = tid % kChunks;
    if (e >= 0) {
      const int t0 = e * kBlock;
      for (int r = tid / kChunks; r < kBlock; r += 128 / kChunks) {
        const bool ok = t0 + r < tk;
        const __nv_bfloat16* ks = ok ? row_ptr(p.k, p.Tk, b, h, t0 + r, p.status) : p.k.ptr;
        const __nv_bfloat16* vs = ok ? row_ptr(p.v, p.Tk, b, h, t0 + r, p.status) : p.v.ptr;
        cp_async16(swz<D>(kbase, r, chunk), ks + (ok ? chunk * 8 : 0), ok ? 16 : 0);
        cp_async16(swz<D>(vbase, r, chunk), vs + (ok ? chunk * 8 : 0), ok ? 16 : 0);
      }
      if (tid < kBlock) sBias[buf * kBlock + tid] = (t0 + tid < tk) ? 0.f : -INFINITY;
    } else {
      const int c0 = (-e - 1) * kBlock;
      for (int r = tid / kChunks; r < kBlock; r += 128 / kChunks) {
        const bool ok = c0 + r < nkb_b;
        const __nv_bfloat16* ks = ok ? kc_bh + (int64_t)(c0 + r) * D + chunk * 8 : p.kc;
        const __nv_bfloat16* vs = ok ? vc_bh + (int64_t)(c0 + r) * D + chunk * 8 : p.vc;
        cp_async16(swz<D>(kbase, r, chunk), ks, ok ? 16 : 0);
        cp_async16(swz<D>(vbase, r, chunk), vs, ok ? 16 : 0);
      }
      if (tid < kBlock) {
        const int c = c0 + tid;
        float bias = -INFINITY;
        if (c < nkb_b && !((sMask[c >> 5] >> (c & 31)) & 1u)) {
          const int len = min(kBlock, tk - c * kBlock);
          bias = log2f((float)len);
        }
        sBias[buf * kBlock + tid] = bias;
      }
    }
  };

  if (ntiles > 0) load_tile(0, 0);
  cp_async_commit();

  // ---- Q fragments (registers) ----
  cp_async_wait<1>();  // the Q group (older than the first tile group) has landed
  __syncthreads();
  uint32_t qf[D / 16][4];
  {
    const uint32_t base = smem_u32(sQ);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      ldsm_x4(swz<D>(base, warp * 16 + (lane & 15), 2 * kk + (lane >> 4)), qf[kk][0], qf[kk][1],
              qf[kk][2], qf[kk][3]);
  }

  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int i = 0; i < ntiles; ++i) {
    const int buf = i & 1;
    if (i + 1 < ntiles) load_tile(i + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const uint32_t kbase = smem_u32(sK + buf * kTile);
    const uint32_t vbase = smem_u32(sV + buf * kTile);
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kp = 0; kp < D / 32; ++kp) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4(swz<D>(kbase, j * 8 + (lane & 7), 4 * kp + (lane >> 3)), r0, r1, r2, r3);
        mma_bf16_16816(s[j], qf[2 * kp], r0, r1);
        mma_bf16_16816(s[j], qf[2 * kp + 1], r2, r3);
      }
    }
    // scale, bias, row max
    const float* bias = sBias + buf * kBlock;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = j * 8 + (lane & 3) * 2;
      const float b0 = bias[col], b1 = bias[col + 1];
      s[j][0] = s[j][0] * p.scale_log2 + b0;
      s[j][1] = s[j][1] * p.scale_log2 + b1;
      s[j][2] = s[j][2] * p.scale_log2 + b0;
      s[j][3] = s[j][3] * p.scale_log2 + b1;
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float u0 = (n0 == -INFINITY) ? 0.f : n0;
    const float u1 = (n1 == -INFINITY) ? 0.f : n1;
    const float a0 = fast_exp2(m0 - u0), a1 = fast_exp2(m1 - u1);
    m0 = n0;
    m1 = n1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = fast_exp2(s[j][0] - u0);
      s[j][1] = fast_exp2(s[j][1] - u0);
      s[j][2] = fast_exp2(s[j][2] - u1);
      s[j][3] = fast_exp2(s[j][3] - u1);
      ps0 += s[j][0] + s[j][1];
      ps1 += s[j][2] + s[j][3];
    }
    l0 = l0 * a0 + ps0;
    l1 = l1 * a1 + ps1;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= a0;
      o[j][1] *= a0;
      o[j][2] *= a1;
      o[j][3] *= a1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dn = 0; dn < D / 16; ++dn) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(swz<D>(vbase, kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, 2 * dn + (lane >> 4)),
                  r0, r1, r2, r3);
        mma_bf16_16816(o[2 * dn], a, r0, r1);
        mma_bf16_16816(o[2 * dn + 1], a, r2, r3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // ---- epilogue ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  {
    const uint32_t base = smem_u32(sQ);
    const int r0 = warp * 16 + (lane >> 2);
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const uint32_t v0 = pack_bf16(o[j][0] * inv0, o[j][1] * inv0);
      const uint32_t v1 = pack_bf16(o[j][2] * inv1, o[j][3] * inv1);
      asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(swz<D>(base, r0, j) + (lane & 3) * 4), "r"(v0));
      asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(swz<D>(base, r0 + 8, j) + (lane & 3) * 4),
                   "r"(v1));
    }
  }
  __syncthreads();
  {
    const int chunk = tid % kChunks;
    for (int r = tid / kChunks; r < kBlock; r += 128 / kChunks) {
      if (q0 + r >= p.Tq) break;
      uint4 val;
      const uint32_t a = swz<D>(smem_u32(sQ), r, chunk);
      asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];\n"
                   : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                   : "r"(a));
      int64_t orow = (int64_t)b * p.Tq + q0 + r;
      if (p.out_idx) {  // scatter: output row out_idx[b * Tq + t]
        orow = __ldg(p.out_idx + orow);
        if (orow < 0 || orow >= p.out_rows) {
          report(p.status, kStatusBadIndex);
          continue;
        }
      }
      __nv_bfloat16* dst = p.out + (orow * p.H + h) * D + chunk * 8;
      *reinterpret_cast<uint4*>(dst) = val;
    }
  }
}

size_t attn_mma_smem_bytes(int D, int nkb) {
  return D == 128 ? MmaSmem<128>::bytes(nkb) : MmaSmem<64>::bytes(nkb);
}

cudaError_t launch_attn_mma(const AttnParams& p, int D, cudaStream_t stream) {
  const size_t smem = attn_mma_smem_bytes(D, p.nkb);
  dim3 grid(p.nqb, p.B * p.H);
  cudaError_t err;
  if (D == 128) {
    err = cudaFuncSetAttribute(attn_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
    if (err != cudaSuccess) return err;
    attn_mma_kernel<128><<<grid, 128, smem, stream>>>(p);
  } else {
    err = cudaFuncSetAttribute(attn_mma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
    if (err != cudaSuccess) return err;
    attn_mma_kernel<64><<<grid, 128, smem, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace solattn

namespace solattn {
cudaError_t launch_attn_sm100(const AttnParams& p, int D, cudaStream_t stream);
bool attn_sm100_supported(const AttnParams& p);

// Every call runs on the tcgen05/TMA kernel except one with more than 4096 key blocks
// (T > 262144 keys), which the int16 tile list of that kernel cannot address: only that size
// reaches this mma.sync kernel.
cudaError_t launch_attention(const AttnParams& p, int D, cudaStream_t stream) {
  if (attn_sm100_supported(p))
    return launch_attn_sm100(p, D, stream);
  return launch_attn_mma(p, D, stream);
}
}  // namespace solattn
