// Grouped packed-ternary expert GEMM on the 5th-generation tensor cores
// (tcgen05, accumulators in tensor memory) for experts with many routed
// tokens: prompt prefill and large batches.
//
// Reference: kernels/ternary_expert.py:240-319 (_ternary_expert_swiglu_kernel)
// and :58-122 (_ternary_expert_gemv_kernel), which the reference runs per
// (token, slot); kernels/ternary_gemv.py:156-258 is its tl.dot GEMM.
//
// Arithmetic: the exact integer contraction of the batch-1 and mma.sync paths
// (the FXA digits of each activation row contracted with the codes, recombined
// exactly, rounded once), so every output equals theirs bit for bit.
//
//   1. fxa_plain_kernel writes, for every routed slot in expert-sorted order
//      (the MoE plan), the slot's activation row as four plain s8 digit rows
//      of K bytes (digit j of X_k = rint(x_k 2^s)) plus the row metadata
//      (shift, rstd, digit totals) -- the same values fxa_prologue produces.
//   2. tgemm_tc_kernel, one CTA per (128 weight rows, expert): for each
//      128-byte K block the threads expand the 2-bit codes of the tile to u8
//      bytes in shared memory (128-byte swizzled, K-major), a tiled TMA load
//      brings the 256 digit rows of the next 64 slots, and one thread issues
//      four tcgen05.mma.kind::i8 (M = 128 codes rows, N = 256 = 64 slots x 4
//      digits, K = 32 bytes each) accumulating u8 x s8 -> s32 in tensor
//      memory; tcgen05.commit releases the stage (3 stages).  The epilogue
//      reads the accumulators with tcgen05.ld (one TMEM lane = one weight
//      row per thread, the four digit sums of a slot in four columns),
//      recombines S = sum_j (C_j - tot_j) 128^j exactly, and applies alpha
//      (and the SwiGLU of the up/gate row pairs) as the mma.sync path does.
//
// Every wait is bounded: a wait that gives up sets bit 1 of the error word,
// waits (bounded) for the CTA's copies and MMAs in flight, frees its tensor
// memory and returns.  Each CTA loads its own tiles from this GPU's memory.
#include "bulk.cuh"
#include "fxa.cuh"
#include "launch.cuh"
#include "tmap.cuh"

namespace mb {

constexpr unsigned kTcBadSlot = 0x80000000u;  // plan list flag: out-of-range expert id
constexpr int kTcMeta = 8;                    // s, rstd bits, tot[0..3], 0, 0
constexpr int kTcStages = 3;
constexpr int kTcARows = 128;                 // MMA M: weight rows per CTA
constexpr int kTcBRows = 256;                 // MMA N: 64 slots x 4 digits
constexpr int kTcSlots = kTcBRows / 4;
constexpr int kTcABytes = kTcARows * 128;     // one 128-byte K block of A
constexpr int kTcBBytes = kTcBRows * 128;
constexpr int kTcStage = kTcABytes + kTcBBytes;
constexpr int kTcCodeSlots = 8;               // code tiles in flight (K blocks ahead)
constexpr int kTcCodeBytes = kTcARows * 32;   // one K block of packed codes: 128 rows x 8 words

// ---------------------------------------------------------------- encode --
// Position p (expert-sorted) encodes input row (list[p] & ~bad) / in_div;
// positions past offsets[n_experts] (slots of other ranks' experts under
// expert parallelism, not listed) are skipped.
template <int XT, int RT, bool RMS>
__global__ void __launch_bounds__(256) fxa_plain_kernel(const void* x, int64_t x_stride, const void* rms_w, float eps,
                                                        int K, const int* offsets, int n_experts,
                                                        const unsigned* list, int in_div, int8_t* digits,
                                                        int* meta) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ FxaBlock fb;
  const int iters = (K + 255) / 256;
  uint2* frag = reinterpret_cast<uint2*>(smem);
  float* xsm = reinterpret_cast<float*>(smem + (size_t)iters * 256 * sizeof(uint2));
  float* wsm = xsm + K;  // RMS: x * w, the encoded values
  const int p = blockIdx.x;
  pdl_wait();
  // the GEMM that follows is released only once these CTAs are done: its
  // CTAs (216 KB of shared memory each) would otherwise take the SMs this
  // multi-wave grid still needs
  if (p >= offsets[n_experts]) {
    pdl_trigger();
    return;
  }
  const int64_t row = (int64_t)(list[p] & ~kTcBadSlot) / in_div;
  const void* xr = static_cast<const char*>(x) + row * x_stride * (XT == kBF16 ? 2 : 4);
  // shift and digit totals exactly as the fragment encoders compute them
  fxa_prologue<XT, RT, RMS, 2, 256>(xr, rms_w, K, eps, 0, iters, xsm, RMS ? wsm : nullptr, frag, fb);
  const int s = fb.s;
  const bool bad = (s == kFxaNonFinite);
  const float* xh = RMS ? wsm : xsm;
  int8_t* d0 = digits + (int64_t)p * 4 * K;
  for (int k = 4 * threadIdx.x; k < K; k += 4 * 256) {
    uint32_t u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) u[i] = static_cast<uint32_t>((bad ? 0 : fxa_enc(xh[k + i], s)) + kFxaOffset);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint32_t*>(d0 + (int64_t)j * K + k) = signed_digits(raw_digits(u[0], u[1], u[2], u[3], j));
  }
  if (threadIdx.x < kTcMeta) {
    const int j = threadIdx.x;
    int v = 0;
    if (j == 0) v = s;
    else if (j == 1) v = __float_as_int(fb.rstd);
    else if (j < 6) v = fb.tot[j - 2];
    meta[(int64_t)p * kTcMeta + j] = v;
  }
  pdl_trigger();
}

// ------------------------------------------------------------ tcgen05 ----
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(unsigned* dst_smem, unsigned ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(unsigned taddr, unsigned ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(unsigned saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// D[tmem] (+)= A x B^T, u8 x s8 -> s32.
__device__ __forceinline__ void umma_i8(unsigned tmem_d, uint64_t da, uint64_t db, unsigned idesc, unsigned accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accum), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(unsigned taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// The 16 two-bit codes of a word (LSB first) as 16 bytes, code i in byte i.
__device__ __forceinline__ uint4 expand_codes16(uint32_t w) {
  const uint32_t t0 = w & 0x33333333u, t1 = (w >> 2) & 0x33333333u;
  const uint32_t e = t0 & 0x0F0F0F0Fu, f = (t0 >> 4) & 0x0F0F0F0Fu;  // codes 4b, 4b+2 in byte b
  const uint32_t g = t1 & 0x0F0F0F0Fu, h = (t1 >> 4) & 0x0F0F0F0Fu;  // codes 4b+1, 4b+3
  const uint32_t lo = __byte_perm(e, g, 0x5140), hi = __byte_perm(f, h, 0x5140);
  const uint32_t lo2 = __byte_perm(e, g, 0x7362), hi2 = __byte_perm(f, h, 0x7362);
  return make_uint4(__byte_perm(lo, hi, 0x5410), __byte_perm(lo, hi, 0x7632), __byte_perm(lo2, hi2, 0x5410),
                    __byte_perm(lo2, hi2, 0x7632));
}

struct TcGemmParams {
  const uint32_t* codes;  // [E, rows, K/16]
  const void* alpha;      // [E, rows]
  const int* offsets;     // [E + 1] positions of each expert in the sorted list
  const unsigned* list;   // [n_pos] slot ids (output rows), kTcBadSlot flagged
  const int* meta;        // [n_pos, 8]
  void* y;
  int* err;
  int64_t y_stride, expert_words, alpha_estride;
  int rows, n_out, K, nwords;
  int use_rstd;           // multiply by the row's rstd (fused input RMSNorm, plain mode)
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
constexpr int kTcExp = 256;  // expander / epilogue threads (warps 0-7)
// Barrier among the expander threads only (the other warps run on).
__device__ __forceinline__ void sync_expanders() { asm volatile("bar.sync 1, 256;\n" ::: "memory"); }
// The same barrier returning the AND of every thread's predicate, so a
// bounded wait's outcome is one decision for all four warps.
__device__ __forceinline__ bool sync_expanders_and(bool v) {
  unsigned r;
  asm volatile(
      "{\n .reg .pred a, b;\n setp.ne.u32 a, %1, 0;\n bar.red.and.pred b, 1, 256, a;\n selp.u32 %0, 1, 0, b;\n}\n"
      : "=r"(r)
      : "r"((unsigned)v)
      : "memory");
  return r != 0;
}

// Roles (352 threads): warps 0-7 expand the codes (thread t: weight row
// t % 128 of the tile, words 4(t / 128) .. +3 of each K block) and run the
// epilogue (TMEM lane group = warp % 4, slot quads split between the two
// warp halves); warp 10 lane 0 streams the packed code tiles from HBM by TMA
// into a ring of 8 K blocks (32 KB in flight per SM hides the DRAM latency);
// warp 8 lane 0 loads the digit tiles; warp 9 lane 0 issues the MMAs.  Per
// code slot: cfull (TMA bytes), cempty (8 expander-warp arrivals); per MMA
// stage: full (TMA bytes), afull (8 expander-warp arrivals), empty
// (tcgen05.commit); per
// chunk of 64 slots: accfull (commit after its last MMA), accempty (256
// epilogue arrivals).  N = 64 x the digit boxes the chunk needs, so decode-
// sized groups (a few slots per expert) run narrow MMAs.  The dependent launch
// is released only after the mainloop: an earlier trigger would let the next
// kernel's CTAs sit on SMs this multi-wave grid still needs.
template <int AT, int OT, bool SWIGLU>
__global__ void __launch_bounds__(352, 1) tgemm_tc_kernel(TcGemmParams p, const __grid_constant__ CUtensorMap tmb,
                                                          const __grid_constant__ CUtensorMap tmc) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* s_gate = reinterpret_cast<float*>(smem + kTcStages * kTcStage);  // [2][64 slots][64 rows]
  unsigned char* codes_s = smem + kTcStages * kTcStage + 2 * kTcSlots * 64 * sizeof(float);  // [8][128][32 B]
  __shared__ uint64_t full[kTcStages], afull[kTcStages], empty[kTcStages], accfull, accempty;
  __shared__ uint64_t cfull[kTcCodeSlots], cempty[kTcCodeSlots];
  __shared__ unsigned s_tmem;
  __shared__ int s_fail;
  __shared__ int s_meta[kTcSlots][kTcMeta];
  __shared__ unsigned s_slot[kTcSlots];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int mt = blockIdx.x, e = blockIdx.y;
  pdl_wait();
  const int first = p.offsets[e], count = p.offsets[e + 1] - first;
  if (count <= 0) {
    pdl_trigger();
    return;
  }

  if (warp == 0) tmem_alloc(&s_tmem, kTcBRows);
  if (tid == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&afull[i], kTcExp / 32);  // one arrival per expander warp
      mbar_init(&empty[i], 1);
    }
    mbar_init(&accfull, 1);
    mbar_init(&accempty, kTcExp);
    for (int i = 0; i < kTcCodeSlots; ++i) {
      mbar_init(&cfull[i], 1);
      mbar_init(&cempty[i], kTcExp / 32);
    }
    s_fail = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = s_tmem;
  const int KB = p.K / 128;
  const int nchunks = (count + kTcSlots - 1) / kTcSlots;
  auto nboxes_of = [&](int c) {  // 64-row digit boxes (16 slots each) chunk c needs
    const int npos = min(kTcSlots, count - kTcSlots * c);
    return (npos + 15) / 16;
  };

  if (warp == 8) {
    // ---------------- TMA producer: digit tiles ----------------
    if (lane == 0) {
      int gi = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int p0 = first + kTcSlots * c, nb = nboxes_of(c);
        for (int kb = 0; kb < KB; ++kb, ++gi) {
          const int st = gi % kTcStages, use = gi / kTcStages;
          if (gi >= kTcStages && !mbar_wait_bounded(&empty[st], (unsigned)((use - 1) & 1))) {
            s_fail = 1;
            atomicOr(p.err, kErrFlagTimeout);
            c = nchunks;
            break;
          }
          unsigned char* B = smem + st * kTcStage + kTcABytes;
          mbar_expect_tx(&full[st], (unsigned)(nb * 8192));
          for (int bx = 0; bx < nb; ++bx) tma_load_2d(B + bx * 8192, &tmb, 128 * kb, 4 * p0 + 64 * bx, &full[st]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 10) {
    // ---------------- TMA producer: packed code tiles ----------------
    if (lane == 0) {
      // tile rows: two boxes of 64 rows (SwiGLU: the up and the gate rows)
      const int rows0 = e * p.rows + (SWIGLU ? 64 * mt : kTcARows * mt);
      const int rows1 = SWIGLU ? e * p.rows + p.n_out + 64 * mt : rows0 + 64;
      const int total = nchunks * KB;
      for (int gc = 0; gc < total; ++gc) {
        const int slot = gc % kTcCodeSlots, use = gc / kTcCodeSlots, kb = gc % KB;
        if (gc >= kTcCodeSlots && !mbar_wait_bounded(&cempty[slot], (unsigned)((use - 1) & 1))) {
          s_fail = 1;
          atomicOr(p.err, kErrFlagTimeout);
          break;
        }
        unsigned char* dst = codes_s + slot * kTcCodeBytes;
        mbar_expect_tx(&cfull[slot], (unsigned)kTcCodeBytes);
        tma_load_2d(dst, &tmc, 8 * kb, rows0, &cfull[slot]);
        tma_load_2d(dst + 64 * 32, &tmc, 8 * kb, rows1, &cfull[slot]);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int gi = 0;
      bool ok = true;
      for (int c = 0; c < nchunks && ok; ++c) {
        const unsigned n = (unsigned)(64 * nboxes_of(c));
        const unsigned idesc = (2u << 4) | (0u << 7) | (1u << 10) | ((n >> 3) << 17) | ((unsigned)(kTcARows >> 4) << 24);
        if (c > 0) ok = mbar_wait_bounded(&accempty, (unsigned)((c - 1) & 1));
        for (int kb = 0; kb < KB && ok; ++kb, ++gi) {
          const int st = gi % kTcStages, use = gi / kTcStages;
          ok = mbar_wait_bounded(&afull[st], (unsigned)(use & 1)) && mbar_wait_bounded(&full[st], (unsigned)(use & 1));
          if (!ok) break;
          tc_fence_after();
          const unsigned sa = smem_u32(smem + st * kTcStage), sb = sa + kTcABytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_i8(tmem, umma_desc_sw128(sa + 32 * kk), umma_desc_sw128(sb + 32 * kk), idesc,
                    (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&accfull);
      }
      if (!ok) {
        s_fail = 1;
        atomicOr(p.err, kErrFlagTimeout);
      }
    }
    __syncwarp();
  } else {
    // ---------------- expanders + epilogue (warps 0-7) ----------------
    const int m = tid & 127, hh = tid >> 7;  // weight row of the tile (= TMEM lane), word half
    int arow;
    bool aok;
    if constexpr (SWIGLU) {  // rows 0-63: up rows n0+r; rows 64-127: gate rows n_out+n0+r
      const int n0 = 64 * mt, r = m & 63;
      aok = n0 + r < p.n_out;
      arow = (m < 64 ? 0 : p.n_out) + n0 + r;
    } else {
      arow = kTcARows * mt + m;
      aok = arow < p.rows;
    }
    const void* alpha_e = static_cast<const char*>(p.alpha) + (int64_t)e * p.alpha_estride * (AT == kBF16 ? 2 : 4);
    const float a_m = aok ? load_f<AT>(alpha_e, arow) : 0.0f;
    char* y = static_cast<char*>(p.y);
    int gi = 0;
    bool ok = true;
    for (int c = 0; c < nchunks && ok; ++c) {
      const int p0 = first + kTcSlots * c, npos = min(kTcSlots, count - kTcSlots * c);
      if (tid < kTcSlots) {
        if (tid < npos) {
          s_slot[tid] = p.list[p0 + tid];
#pragma unroll
          for (int j = 0; j < kTcMeta; ++j) s_meta[tid][j] = p.meta[(int64_t)(p0 + tid) * kTcMeta + j];
        } else {
          s_slot[tid] = 0xffffffffu;
        }
      }
      for (int kb = 0; kb < KB; ++kb, ++gi) {
        const int st = gi % kTcStages, use = gi / kTcStages;
        const int cs = gi % kTcCodeSlots, cuse = gi / kTcCodeSlots;
        const bool ready = (gi < kTcStages || mbar_wait_bounded(&empty[st], (unsigned)((use - 1) & 1))) &&
                           mbar_wait_bounded(&cfull[cs], (unsigned)(cuse & 1));
        if (!sync_expanders_and(ready)) {
          ok = false;
          break;
        }
        const uint4 wa = aok ? *reinterpret_cast<const uint4*>(codes_s + cs * kTcCodeBytes + m * 32 + hh * 16)
                             : make_uint4(0, 0, 0, 0);
        unsigned char* arow_s = smem + st * kTcStage + (m >> 3) * 1024 + (m & 7) * 128;
        const uint32_t ws[4] = {wa.x, wa.y, wa.z, wa.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int u = 4 * hh + i;
          *reinterpret_cast<uint4*>(arow_s + ((u ^ (m & 7)) << 4)) = expand_codes16(ws[i]);
        }
        fence_proxy_async_smem();  // the tensor core reads these bytes through the async proxy
        // One arrival per warp (not per thread) on each barrier: the warp's
        // code reads were consumed by the expansion above and its stores are
        // ordered before lane 0's release by the warp barrier.
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&cempty[cs]);
          mbar_arrive(&afull[st]);
        }
      }
      if (!ok || !sync_expanders_and(mbar_wait_bounded(&accfull, (unsigned)(c & 1)))) {
        ok = false;
        break;
      }
      tc_fence_after();  // (the reduction above also made s_slot / s_meta visible)
      if (c == nchunks - 1) pdl_trigger();
      for (int pb = hh; 4 * pb < npos; pb += 2) {
        uint32_t r[16];
        tmem_ld16(tmem + ((unsigned)(32 * (warp & 3)) << 16) + (unsigned)(16 * pb), r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int idx = 4 * pb + i;
          if (idx < npos) {
            const int* ms = s_meta[idx];
            const int c0 = (int)r[4 * i] - ms[2], c1 = (int)r[4 * i + 1] - ms[3];
            const int c2 = (int)r[4 * i + 2] - ms[4], c3 = (int)r[4 * i + 3] - ms[5];
            const long long S = ((long long)c0 + 128LL * c1) + 16384LL * ((long long)c2 + 128LL * c3);
            const unsigned slot = s_slot[idx];
            const int sh = ms[0];
            const bool nan_out = (sh == kFxaNonFinite) || (slot & kTcBadSlot);
            float v = nan_out ? __int_as_float(0x7fc00000) : fxa_value(S, sh);
            if (!SWIGLU && p.use_rstd) v = __fmul_rn(v, __int_as_float(ms[1]));
            v = __fmul_rn(v, a_m);
            if constexpr (SWIGLU) {
              if (m >= 64) s_gate[idx * 64 + (m - 64)] = v;
              else s_gate[kTcSlots * 64 + idx * 64 + m] = v;  // up values after the gate block
            } else if (aok) {
              store_f<OT>(y + (int64_t)(slot & ~kTcBadSlot) * p.y_stride * (OT == kBF16 ? 2 : 4), arow, v);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&accempty);  // this thread's TMEM reads are done
      if constexpr (SWIGLU) {
        sync_expanders();
        for (int q = tid; q < npos * 64; q += kTcExp) {
          const int idx = q >> 6, nn = q & 63;
          const int n = 64 * mt + nn;
          if (n < p.n_out) {
            float up = s_gate[kTcSlots * 64 + idx * 64 + nn], gate = s_gate[idx * 64 + nn];
            up = fminf(fmaxf(up, -7.0f), 7.0f);
            gate = fminf(gate, 7.0f);
            const unsigned slot = s_slot[idx];
            // an out-of-range expert id gives a NaN row (the clamps would turn NaN into -49)
            store_f<OT>(y + (int64_t)(slot & ~kTcBadSlot) * p.y_stride * (OT == kBF16 ? 2 : 4), n,
                        (slot & kTcBadSlot) ? __int_as_float(0x7fc00000)
                                            : __fmul_rn(__fmul_rn(up, gate), msigmoid(gate)));
          }
        }
      }
      sync_expanders();  // staging and slot tables free for the next chunk
    }
    if (!ok) {
      s_fail = 1;
      atomicOr(p.err, kErrFlagTimeout);
    }
  }
  __syncthreads();
  pdl_trigger();  // (a no-op where the epilogue already released it)
  if (s_fail) {
    // give the copies and MMAs this CTA issued time to land (about a
    // millisecond, bounded) before its shared and tensor memory go
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcBRows);
  }
}

}  // namespace mb

using namespace mb;

extern "C" int64_t maple_ternary_grouped_gemm_tc_workspace_bytes(int64_t n_slots, int64_t k) {
  if (n_slots < 0 || k <= 0) return -1;
  const int64_t dig = (n_slots * 4 * k + 255) / 256 * 256;
  return dig + (n_slots * kTcMeta * 4 + 255) / 256 * 256;
}

extern "C" int maple_ternary_grouped_gemm_tc(const void* x, int x_dtype, int64_t in_rows, int64_t k,
                                             int64_t x_row_stride, const uint32_t* codes, int64_t n_experts,
                                             int64_t code_rows, const void* alpha, int alpha_dtype,
                                             const int32_t* offsets, const uint32_t* list, int64_t n_slots,
                                             int64_t in_div, int swiglu, const void* rms_w, int rms_dtype,
                                             float eps, void* y, int y_dtype, int64_t y_row_stride,
                                             void* workspace, int64_t workspace_bytes, int* err, void* stream) {
  if (in_rows < 0 || n_slots < 0 || n_experts <= 0 || code_rows <= 0 || in_div <= 0) return kErrShape;
  if (k <= 0 || k % 128 != 0 || k > 8192) return kErrShape;
  if (n_slots == 0) return kOk;
  if (swiglu && code_rows % 2 != 0) return kErrShape;
  if (!x || !codes || !alpha || !offsets || !list || !y || !err || !workspace) return kErrShape;
  if ((n_slots - 1) / in_div >= in_rows) return kErrBounds;
  if (x_dtype != kBF16 && x_dtype != kF32) return kErrDtype;
  if ((alpha_dtype != kBF16 && alpha_dtype != kF32) || (y_dtype != kBF16 && y_dtype != kF32)) return kErrDtype;
  if (rms_w && rms_dtype != kBF16 && rms_dtype != kF32) return kErrDtype;
  if (rms_w && swiglu) return kErrShape;  // the fused input norm is for plain (dense) GEMMs
  if (workspace_bytes < maple_ternary_grouped_gemm_tc_workspace_bytes(n_slots, k)) return kErrWorkspace;
  if ((reinterpret_cast<uintptr_t>(codes) | reinterpret_cast<uintptr_t>(workspace)) & 255) return kErrAlign;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || ((x_row_stride * (x_dtype == kBF16 ? 2 : 4)) & 15)) return kErrAlign;
  if (n_experts > 65535 || code_rows > (1LL << 30) || n_slots * 4 > (1LL << 31) - 1) return kErrShape;
  int8_t* digits = static_cast<int8_t*>(workspace);
  int* meta = reinterpret_cast<int*>(static_cast<char*>(workspace) + (n_slots * 4 * k + 255) / 256 * 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int K = (int)k, iters = (K + 255) / 256;
  const size_t esmem = (size_t)iters * 256 * sizeof(uint2) + (size_t)(rms_w ? 2 : 1) * K * sizeof(float);
  cudaError_t e = cudaSuccess;
  {
    void (*kern)(const void*, int64_t, const void*, float, int, const int*, int, const unsigned*, int, int8_t*,
                 int*);
    if (!rms_w) kern = x_dtype == kBF16 ? fxa_plain_kernel<kBF16, kF32, false> : fxa_plain_kernel<kF32, kF32, false>;
    else if (rms_dtype == kBF16)
      kern = x_dtype == kBF16 ? fxa_plain_kernel<kBF16, kBF16, true> : fxa_plain_kernel<kF32, kBF16, true>;
    else kern = x_dtype == kBF16 ? fxa_plain_kernel<kBF16, kF32, true> : fxa_plain_kernel<kF32, kF32, true>;
    if (esmem > 32 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)esmem);
    if (e == cudaSuccess)
      e = launch_k(kern, dim3((unsigned)n_slots), dim3(256), esmem, st, x, x_row_stride, rms_w, eps, K, offsets,
                   (int)n_experts, list, (int)in_div, digits, meta);
    if (e != cudaSuccess) return kErrCuda;
  }
  CUtensorMap tmb;
  CUtensorMap tmc;
  if (!tmap_2d(digits, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k, 4 * n_slots, 128, 64, true, &tmb) ||
      !tmap_2d(codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, k / 16, n_experts * code_rows, 8, 64, false, &tmc))
    return kErrCuda;
  TcGemmParams p{};
  p.codes = codes; p.alpha = alpha; p.offsets = offsets; p.list = list; p.meta = meta; p.y = y; p.err = err;
  p.y_stride = y_row_stride; p.expert_words = code_rows * (k / 16); p.alpha_estride = code_rows;
  p.rows = (int)code_rows; p.n_out = swiglu ? (int)(code_rows / 2) : (int)code_rows;
  p.K = K; p.nwords = (int)(k / 16); p.use_rstd = rms_w != nullptr;
  const int tiles = swiglu ? (p.n_out + 63) / 64 : (p.rows + kTcARows - 1) / kTcARows;
  const dim3 grid((unsigned)tiles, (unsigned)n_experts);
  const size_t gsmem = (size_t)kTcStages * kTcStage + 2 * (size_t)kTcSlots * 64 * sizeof(float) +
                       (size_t)kTcCodeSlots * kTcCodeBytes + 1024;
#define MB_TCG(AT_, OT_, SW_)                                                                                  \
  do {                                                                                                         \
    auto kern = tgemm_tc_kernel<AT_, OT_, SW_>;                                                                \
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsmem);                   \
    if (e == cudaSuccess) e = launch_k(kern, grid, dim3(352), gsmem, st, p, tmb, tmc);                        \
  } while (0)
#define MB_TCG_SW(AT_, OT_) \
  do {                      \
    if (swiglu) MB_TCG(AT_, OT_, true); else MB_TCG(AT_, OT_, false); \
  } while (0)
  if (alpha_dtype == kBF16) {
    if (y_dtype == kBF16) MB_TCG_SW(kBF16, kBF16); else MB_TCG_SW(kBF16, kF32);
  } else {
    if (y_dtype == kBF16) MB_TCG_SW(kF32, kBF16); else MB_TCG_SW(kF32, kF32);
  }
#undef MB_TCG_SW
#undef MB_TCG
  return e == cudaSuccess ? kOk : kErrCuda;
}
