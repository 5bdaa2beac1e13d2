// Prefill / bidirectional attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Reference semantics: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/layers/Attention.java:245-280,
// 308-396 (causal prefill over paged KV with a cached prefix, sliding window, soft-cap) and
// BidirectionalAttention.java:71-145 (BERT, no mask); the online-softmax formulation is the usual flash
// attention one.
//
// One CTA per (tile of 128 query rows, KV head, sequence).  A query row is a (token, head-of-the-GQA-group)
// pair: the G heads that share a KV head are packed into the MMA's 128 rows, so one K/V tile serves all of
// them.  Per KV tile of BN keys:
//   S  = Q K^T        tcgen05.mma, A = Q (shared memory, K-major), B = K tile (shared memory, K-major), D in TMEM
//   P  = softmax(S)   256 softmax threads, two per query row (TMEM lane), each on half of the tile's keys:
//                     tcgen05.ld, mask, online max (exchanged between the halves), exp2, row sum; P goes back
//                     as bf16 into the first BN/2 columns of the same TMEM buffer
//   O += P V          tcgen05.mma with A = P read from TMEM and B = V tile (shared memory, MN-major: the cache
//                     stores keys as rows with head_dim contiguous), fp32 O accumulator in TMEM
// S is double-buffered in TMEM (S of tile j+1 is computed while the softmax threads work on tile j).  The max
// is only moved (and O, l rescaled through a TMEM load/store of the row) when a tile's row max exceeds the
// one in use by more than 2^8; otherwise exponentials are taken against the stale max, which keeps P <= 256
// and the final O / l exact.
// Warps: 0 / 3 TMA producers (K ring / V ring), 1 MMA issuer (lane 0), 2 MMA waiter (does every mbarrier wait of the issuer
// and hands over through a named barrier: an mbarrier wait in the issuing thread right after a batch of
// tcgen05.mma stalls until the batch drains), 4-11 softmax + epilogue.  Every wait is bounded.
#pragma once
#include "common.cuh"

namespace {

template <int HD>
struct TcAttnCfg {
  static constexpr int BN = HD == 256 ? 64 : 128;     // keys per tile
  // separate K and V rings: a K tile is free once its S MMA is done (so K runs KS tiles ahead of the MMAs),
  // a V tile once its PV MMA is done
  static constexpr int KS = HD == 64 ? 4 : HD == 256 ? 2 : 3;
  static constexpr int VS = HD == 64 ? 4 : 2;
  static constexpr int KBOX = BN * 128;               // one 64-dim box of a K or V tile, bytes
  static constexpr int KTILE = (HD / 64) * KBOX;      // K (or V) tile, bytes
  static constexpr int QBOX = 128 * 128;              // 128 query rows x 64 dims, bytes
  static constexpr int QTILE = (HD / 64) * QBOX;
  static constexpr uint32_t O_COL = 2 * BN;           // TMEM: S buffers [0, 2 BN), O [2 BN, 2 BN + HD)
  static_assert(O_COL + HD <= 512, "TMEM plan");
  static constexpr size_t smem() { return 1024 + QTILE + (size_t)(KS + VS) * KTILE + 256 + 6 * 128 * 4; }
};

__device__ __forceinline__ void tca_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tca_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tca_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// Named barrier 3 over the 256 softmax threads; returns how many passed a non-zero flag.
__device__ __forceinline__ int __syncthreads_count_named(int flag) {
  int n;
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.popc.u32 %0, 3, 256, p;\n\t}"
               : "=r"(n)
               : "r"(flag)
               : "memory");
  return n;
}
__device__ __forceinline__ void tca_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D(tmem) (+)= A(tmem) * B(smem desc), kind::f16 (bf16 per the instruction descriptor)
__device__ __forceinline__ void tca_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory descriptor of an MN-major operand in the 128-byte swizzle TMA writes for a box of 64 elements
// (128 B) x rows: rows run along K (8-row swizzle atoms 1024 B apart: SBO), 64-element blocks along MN are
// ``mn_stride`` bytes apart (LBO).  Checked on B200 against a CPU product.
__device__ __forceinline__ uint64_t tca_desc_mn_sw128(uint32_t addr, uint32_t mn_stride) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((mn_stride >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Named barrier 2 between the MMA issuer warp and its waiter warp, AND-reducing an ok flag.
__device__ __forceinline__ bool tca_handoff(int ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, 2, 64, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(ok)
      : "memory");
  return r != 0;
}

// HD: the head dim the tiles are laid out for; HDR (<= HD): the model's head dim.  HDR 32 (BERT-small shapes)
// runs in 64-wide tiles: Q's upper 32 dims are zero, so the neighbouring head's K dims that the 64-wide K box
// brings along add nothing to S, and the matching upper half of O is never written out (contiguous K/V only).
template <int HD, int HDR = HD>
__global__ void __launch_bounds__(384, 1) prefill_tc_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const bf16* __restrict__ q,
    long q_tok_stride, bf16* __restrict__ out, long o_tok_stride, const int* __restrict__ cu_q,
    const int* __restrict__ cu_k, const int* __restrict__ block_tables, int bt_stride, int paged, int nq, int nkv,
    int block_size, float scale, float softcap, int window, int causal, int* err) {
  using C = TcAttnCfg<HD>;
  constexpr int BN = C::BN, KS = C::KS, VS = C::VS;
  constexpr uint32_t IDESC_S = nvb::idesc_bf16_f32(128, BN);
  constexpr uint32_t IDESC_PV = nvb::idesc_bf16_f32(128, HD) | (1u << 16);  // B (V) MN-major
  nvb::pdl_wait();
  nvb::pdl_trigger();
  const int qtile = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const int G = nq / nkv;
  const int TPT = 128 / G;  // tokens per query tile
  const int q0 = cu_q[seq], qlen = cu_q[seq + 1] - q0;
  const int k0 = cu_k[seq], klen = cu_k[seq + 1] - k0;
  const int tok_begin = qtile * TPT;
  if (tok_begin >= qlen) return;
  const int tok_end = min(tok_begin + TPT, qlen);
  const int pos_lo = klen - qlen + tok_begin, pos_hi = klen - qlen + tok_end - 1;
  const int key_end = causal ? min(klen, pos_hi + 1) : klen;
  const int key_begin = (window > 0 && causal) ? max(0, pos_lo - window + 1) : 0;
  const int t_begin = key_begin / BN;
  const int nt = key_end > key_begin ? (key_end + BN - 1) / BN - t_begin : 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* qs = smem;
  uint8_t* kring = smem + C::QTILE;                 // KS K tiles
  uint8_t* vring = kring + (size_t)KS * C::KTILE;   // VS V tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(vring + (size_t)VS * C::KTILE);
  uint64_t* k_full = bars;
  uint64_t* k_free = k_full + KS;
  uint64_t* v_full = k_free + KS;
  uint64_t* v_free = v_full + VS;
  uint64_t* s_full = v_free + VS;   // [2]
  uint64_t* p_full = s_full + 2;    // [2]
  uint64_t* s_free = p_full + 2;    // [2]
  uint64_t* o_done = s_free + 2;    // one phase per PV
  uint64_t* o_final = o_done + 1;
  uint64_t* q_full = o_final + 1;
  uint8_t* smem_extra = reinterpret_cast<uint8_t*>(bars) + 256;  // row-max exchange and row sums (4 KB)
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < KS; ++s) {
      nvb::mbar_init(&k_full[s], 1);
      nvb::mbar_init(&k_free[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      nvb::mbar_init(&v_full[s], 1);
      nvb::mbar_init(&v_free[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      nvb::mbar_init(&s_full[b], 1);
      nvb::mbar_init(&p_full[b], 8);
      nvb::mbar_init(&s_free[b], 1);
    }
    nvb::mbar_init(o_done, 1);
    nvb::mbar_init(o_final, 1);
    nvb::mbar_init(q_full, 8);
    nvb::fence_mbar_init();
  }
  if (warp == 1) {
    nvb::tmem_alloc(&tmem_base_sh, 512);
    nvb::tmem_relinquish();
  }
  nvb::tc_fence_before();
  __syncthreads();
  nvb::tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0 || warp == 3) {
    // ------------------------------------------------------------------ producers: K ring (warp 0), V ring (warp 3)
    const bool is_k = warp == 0;
    if (lane == 0 && nt > 0) {
      const CUtensorMap* map = is_k ? &kmap : &vmap;
      nvb::tma_prefetch_desc(map);
      const int NS = is_k ? KS : VS;
      uint8_t* ringp = is_k ? kring : vring;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* freeb = is_k ? k_free : v_free;
      const int head = is_k ? nq + kvh : nq + nkv + kvh;
      const int* bt = block_tables != nullptr ? block_tables + (long)seq * bt_stride : nullptr;
      int i = 0;
      bool ok = true;
      for (; i < nt; ++i) {
        const int s = i % NS;
        if (i >= NS && !nvb::mbar_wait(&freeb[s], ((i / NS) & 1) ^ 1, err, &abort_flag)) {
          ok = false;
          break;
        }
        const int tok = (t_begin + i) * BN;
        uint8_t* dst = ringp + (size_t)s * C::KTILE;
        nvb::mbar_arrive_expect_tx(&full[s], C::KTILE);
        if (paged) {
          const int row = (bt[tok / block_size] * nkv + kvh) * block_size + (tok % block_size);
#pragma unroll
          for (int j = 0; j < HD / 64; ++j) nvb::tma_load_2d(dst + j * C::KBOX, map, &full[s], j * 64, row);
        } else if constexpr (HDR == HD) {
#pragma unroll
          for (int j = 0; j < HD / 64; ++j) nvb::tma_load_3d(dst + j * C::KBOX, map, &full[s], j * 64, head, k0 + tok);
        } else {
          // 2-D map over packed qkv rows: one 64-wide box from this head's first dim (zero fill past the row end)
          nvb::tma_load_2d(dst, map, &full[s], head * HDR, k0 + tok);
        }
      }
      if (!ok)  // bounded drain of copies that may still be landing
        for (int j = (i > NS ? i - NS : 0); j < i; ++j) nvb::mbar_wait(&full[j % NS], (j / NS) & 1, nullptr, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    bool ok = nt > 0 && tca_handoff(1);  // Q and K tile 0 are in shared memory
    if (ok) {
      nvb::tc_fence_after();
      if (lane == 0) {
        // S of tile j into TMEM buffer j & 1
        auto issue_s = [&](int j) {
          const uint32_t ka = nvb::smem_u32(kring + (size_t)(j % KS) * C::KTILE);
          const uint32_t qa = nvb::smem_u32(qs);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            nvb::tc_mma_f16(tmem + (uint32_t)(j & 1) * BN,
                            nvb::sdesc_kmajor_sw128(qa + (kk >> 2) * C::QBOX + (kk & 3) * 32),
                            nvb::sdesc_kmajor_sw128(ka + (kk >> 2) * C::KBOX + (kk & 3) * 32), IDESC_S,
                            kk > 0 ? 1u : 0u);
          nvb::tc_commit(&s_full[j & 1]);
          nvb::tc_commit(&k_free[j % KS]);
        };
        issue_s(0);
      }
      __syncwarp();
    }
    for (int j = 0; ok && j < nt; ++j) {
      if (j + 1 < nt) {
        ok = tca_handoff(1);  // K tile j + 1 landed, S buffer (j + 1) & 1 free
        if (!ok) break;
        nvb::tc_fence_after();
        if (lane == 0) {
          const int jj = j + 1;
          const uint32_t ka = nvb::smem_u32(kring + (size_t)(jj % KS) * C::KTILE);
          const uint32_t qa = nvb::smem_u32(qs);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            nvb::tc_mma_f16(tmem + (uint32_t)(jj & 1) * BN,
                            nvb::sdesc_kmajor_sw128(qa + (kk >> 2) * C::QBOX + (kk & 3) * 32),
                            nvb::sdesc_kmajor_sw128(ka + (kk >> 2) * C::KBOX + (kk & 3) * 32), IDESC_S,
                            kk > 0 ? 1u : 0u);
          nvb::tc_commit(&s_full[jj & 1]);
          nvb::tc_commit(&k_free[jj % KS]);
        }
        __syncwarp();
      }
      ok = tca_handoff(1);  // P of tile j in TMEM (O rescaled), V tile j landed
      if (!ok) break;
      nvb::tc_fence_after();
      if (lane == 0) {
        const uint32_t va = nvb::smem_u32(vring + (size_t)(j % VS) * C::KTILE);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          tca_mma_ts(tmem + C::O_COL, tmem + (uint32_t)(j & 1) * BN + kk * 8,
                     tca_desc_mn_sw128(va + kk * 2048, C::KBOX), IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        nvb::tc_commit(o_done);
        nvb::tc_commit(&v_free[j % VS]);
        nvb::tc_commit(&s_free[j & 1]);
        if (j == nt - 1) nvb::tc_commit(o_final);
      }
      __syncwarp();
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ MMA waiter
    if (nt > 0) {
      int okl = 1;
      if (lane == 0)
        okl = (nvb::mbar_wait(q_full, 0, err, &abort_flag) && nvb::mbar_wait(&k_full[0], 0, err, &abort_flag)) ? 1 : 0;
      bool ok = tca_handoff(__shfl_sync(0xffffffffu, okl, 0));
      for (int j = 0; ok && j < nt; ++j) {
        if (j + 1 < nt) {
          const int jj = j + 1;
          okl = 1;
          if (lane == 0) {
            okl = nvb::mbar_wait(&k_full[jj % KS], (jj / KS) & 1, err, &abort_flag) ? 1 : 0;
            if (okl && jj >= 2) okl = nvb::mbar_wait(&s_free[jj & 1], ((jj >> 1) - 1) & 1, err, &abort_flag) ? 1 : 0;
          }
          ok = tca_handoff(__shfl_sync(0xffffffffu, okl, 0));
          if (!ok) break;
        }
        okl = 1;
        if (lane == 0)
          okl = (nvb::mbar_wait(&p_full[j & 1], (j >> 1) & 1, err, &abort_flag) &&
                 nvb::mbar_wait(&v_full[j % VS], (j / VS) & 1, err, &abort_flag)) ? 1 : 0;
        ok = tca_handoff(__shfl_sync(0xffffffffu, okl, 0));
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax + epilogue (warps 4-11)
    // warps w and w + 4 share the TMEM lane quarter w & 3 (query rows) and split each S tile's columns: half 0
    // takes keys [0, BN/2), half 1 [BN/2, BN); the halves exchange row maxima through shared memory once per
    // tile, rescale their own half of O, and sum their row sums at the end
    constexpr int HB = BN / 2;          // S columns per half
    constexpr int PC = BN / 4;          // packed P columns per half
    constexpr int OH = HD / 2;          // O columns per half
    const int quarter = warp & 3, half = (warp - 4) >> 2, r = quarter * 32 + lane;
    const int st8 = tid - 128;
    float* xmax = reinterpret_cast<float*>(smem_extra);        // [2 tile parities][2 halves][128 rows]
    float* lsum = xmax + 2 * 2 * 128;                            // [2 halves][128 rows]
    // Q tile -> shared memory in the 128-byte swizzle the MMA reads (rows past the sequence are zero)
    for (int idx = st8; idx < 128 * (HD / 8); idx += 256) {
      const int rr = idx / (HD / 8), c = idx % (HD / 8);  // c: 16-byte chunk of the (padded) row
      const int jt = tok_begin + rr / G;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (jt < qlen && c * 8 < HDR)
        v = *reinterpret_cast<const uint4*>(q + (long)(q0 + jt) * q_tok_stride + (kvh * G + rr % G) * HDR + c * 8);
      *reinterpret_cast<uint4*>(qs + (c >> 3) * C::QBOX + nvb::swz128(rr, c & 7)) = v;
    }
    nvb::fence_proxy_async();
    __syncwarp();
    if (lane == 0) nvb::mbar_arrive(q_full);

    const int jt = tok_begin + r / G;
    const bool rvalid = jt < qlen;
    const int rpos = klen - qlen + jt;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    float m_used = -INFINITY, l = 0.f;
    const float sl2 = scale * kLog2e;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int b = j & 1;
      int okw = 1;
      if (lane == 0) okw = nvb::mbar_wait(&s_full[b], (j >> 1) & 1, err, &abort_flag) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0);
      // every softmax warp reaches the exchange barrier below, ok or not, so none waits there for ever
      nvb::tc_fence_after();
      float s[HB];
      if (okw) {
        uint32_t u[HB];
#pragma unroll
        for (int c = 0; c < HB; c += 32)
          tca_ld32(lane_base + (uint32_t)b * BN + half * HB + c, *reinterpret_cast<uint32_t(*)[32]>(u + c));
        nvb::tmem_ld_wait();
        nvb::reg_fence<HB>(u);
#pragma unroll
        for (int e = 0; e < HB; ++e) s[e] = __uint_as_float(u[e]);
      } else {
#pragma unroll
        for (int e = 0; e < HB; ++e) s[e] = 0.f;
      }
      const int key0 = (t_begin + j) * BN + half * HB;
      // a half-tile every key of which this row may see skips the per-key mask
      const bool whole = rvalid && key0 + HB <= klen &&
                         (!causal || (key0 + HB - 1 <= rpos && (window <= 0 || key0 > rpos - window)));
      float mt = -INFINITY;
      if (whole && softcap <= 0.f) {
#pragma unroll
        for (int e = 0; e < HB; ++e) {
          s[e] *= sl2;
          mt = fmaxf(mt, s[e]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < HB; ++e) {
          const int key = key0 + e;
          float x = softcap > 0.f ? apply_cap(s[e] * scale, softcap) * kLog2e : s[e] * sl2;
          bool valid = rvalid && key < klen;
          if (causal) valid = valid && key <= rpos && (window <= 0 || key > rpos - window);
          if (!valid) x = -INFINITY;
          s[e] = x;
          mt = fmaxf(mt, x);
        }
      }
      xmax[(b * 2 + half) * 128 + r] = mt;
      const int all_ok = __syncthreads_count_named(okw && ok);
      if (all_ok != 256) {
        ok = false;
        break;
      }
      mt = fmaxf(mt, xmax[(b * 2 + (half ^ 1)) * 128 + r]);
      float new_m = m_used;
      bool need = false;
      if (mt > -INFINITY) {
        if (m_used == -INFINITY) {
          new_m = mt;  // the O row is still zero: nothing to rescale
        } else if (mt > m_used + 8.f) {
          new_m = mt;
          need = true;
        }
      }
      if (__any_sync(0xffffffffu, need)) {
        // O must hold P_{j-1} V_{j-1} before it is rescaled (j >= 1 here: some earlier tile set m_used)
        // a failed wait is reported at the next exchange barrier, which every softmax warp still reaches
        okw = 1;
        if (lane == 0) okw = nvb::mbar_wait(o_done, (j - 1) & 1, err, &abort_flag) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, okw, 0)) ok = false;
        nvb::tc_fence_after();
        const float f = need ? exp2f(m_used - new_m) : 1.f;
#pragma unroll 1
        for (int c = 0; ok && c < OH; c += 32) {
          uint32_t u[32];
          tca_ld32(lane_base + C::O_COL + half * OH + c, u);
          nvb::tmem_ld_wait();
          nvb::reg_fence<32>(u);
#pragma unroll
          for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * f);
          tca_st32(lane_base + C::O_COL + half * OH + c, u);
        }
        tca_st_wait();
      }
      if (need) l *= exp2f(m_used - new_m);
      m_used = new_m;
      // P (bf16 pairs) of this half over packed columns [half * PC, half * PC + PC) of the S buffer
      float rs = 0.f;
      uint32_t u[PC];
#pragma unroll
      for (int e = 0; e < PC; ++e) {
        const float p0 = m_used == -INFINITY ? 0.f : exp2f(s[2 * e] - m_used);
        const float p1 = m_used == -INFINITY ? 0.f : exp2f(s[2 * e + 1] - m_used);
        rs += p0 + p1;
        u[e] = nvb::pack_bf16x2(p0, p1);
      }
#pragma unroll
      for (int c = 0; c < PC; c += 16) tca_st16(lane_base + (uint32_t)b * BN + half * PC + c, *reinterpret_cast<uint32_t(*)[16]>(u + c));
      l += rs;
      tca_st_wait();
      nvb::tc_fence_before();
      __syncwarp();
      if (lane == 0) nvb::mbar_arrive(&p_full[b]);
    }
    // epilogue: O / l, bf16 rows (rows past the sequence are not written)
    int okw = ok ? 1 : 0;
    if (okw && nt > 0 && lane == 0) okw = nvb::mbar_wait(o_final, 0, err, &abort_flag) ? 1 : 0;
    okw = __shfl_sync(0xffffffffu, okw, 0);
    lsum[half * 128 + r] = l;
    const int all_ok = __syncthreads_count_named(okw);
    if (all_ok == 256) {
      nvb::tc_fence_after();
      const float lt = l + lsum[(half ^ 1) * 128 + r];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      bf16* dst = out + (long)(q0 + jt) * o_tok_stride + (kvh * G + r % G) * HDR;
#pragma unroll 1
      for (int c = half * OH; c < half * OH + OH; c += 32) {
        if (c >= HDR) break;  // the zero-padded upper dims of a narrow head are not output
        uint32_t u[32];
        if (nt > 0) {
          tca_ld32(lane_base + C::O_COL + c, u);
          nvb::tmem_ld_wait();
          nvb::reg_fence<32>(u);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) u[e] = 0u;
        }
        if (rvalid) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            w.x = nvb::pack_bf16x2(__uint_as_float(u[e]) * inv, __uint_as_float(u[e + 1]) * inv);
            w.y = nvb::pack_bf16x2(__uint_as_float(u[e + 2]) * inv, __uint_as_float(u[e + 3]) * inv);
            w.z = nvb::pack_bf16x2(__uint_as_float(u[e + 4]) * inv, __uint_as_float(u[e + 5]) * inv);
            w.w = nvb::pack_bf16x2(__uint_as_float(u[e + 6]) * inv, __uint_as_float(u[e + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c + e) = w;
          }
        }
      }
    }
  }
  nvb::tc_fence_before();
  __syncthreads();
  nvb::tc_fence_after();
  if (warp == 1) nvb::tmem_dealloc(tmem, 512);
}

}  // namespace
