// Two-Q-tile ("ping-pong") variant of fa_tc_kernel for head_dim 128.
// Included by fa_tc.cu inside its anonymous namespace (shares FaParams,
// fast_exp2, sw_off and the timeline buffer).
//
// One CTA owns 256 query rows of one (sequence, KV head): tile A = rows
// 0-127, tile B = rows 128-255, GQA-packed as in fa_tc_kernel (row r ->
// token t0 + r / G, head kvh * G + r % G); both tiles share every K / V tile,
// so each key tile is loaded once for 256 rows. Eleven warps:
//   warp 0      producer: Q (four boxes) once, then the K tiles
//   warp 1      TMEM owner + MMA issuer
//   warps 2-5   softmax of tile A, one row per thread
//   warp 6      producer: the V tiles
//   warps 7-10  softmax of tile B
// so every SM sub-partition holds one softmax warp of each tile and can issue
// from one while the other waits on a dependency.
// TMEM: S_A | S_B | O_A | O_B, 128 columns each. P (bf16 pairs, 64 columns)
// is written over the first half of its own S buffer after that S has been
// read. Per key tile j the MMA issuer runs PV_A(j), S_A(j+1), PV_B(j),
// S_B(j+1): while one softmax group works on its tile, the tensor core works
// for the other. A commit tracks every earlier MMA of the issuer, so when a
// softmax group sees S_X(j) ready, PV_X(j-1) has completed and O_X stays
// untouched until the group releases P_X(j): the O correction needs no other
// wait. Because P overwrites S, each tile takes its row max in a first pass
// over S and the exponentials in a second; O is rescaled only when a row's
// max grows by more than 2^8 over the max its exponentials use.
// K / V stream through a 2-stage ring (Q takes 64 KB of shared memory).

// 2^x for a pair on the FMA / integer pipes, taking load off the
// multi-function unit: x is clamped to >= -125; adding 1.5 * 2^23 rounds x to
// the nearest integer n (the sum's low mantissa bits hold n: the standard
// magic-constant rounding), f = x - n lies in [-0.5, 0.5]; 2^f comes from a
// degree-3 polynomial fitted for this kernel (max relative error 7.5e-5, far
// below the bf16 rounding of P) and 2^n is applied by adding n to the
// exponent field (the construction of N. Schraudolph, "A fast, compact
// approximation of the exponential function", Neural Computation 11(4),
// 1999). p in [0.70, 1.42] and n >= -125 keep the exponent field positive;
// masked scores (-inf) clamp to 2^-125, which P's bf16 keeps as ~2.4e-38.
__device__ __forceinline__ void exp2_fma_pair(float& a, float& b) {
  a = fmaxf(a, -125.f);
  b = fmaxf(b, -125.f);
  const uint64_t xv = f32x2_pack(a, b);
  const uint64_t t = f32x2_add(xv, f32x2_pack(12582912.f, 12582912.f));
  const uint64_t n = f32x2_add(t, f32x2_pack(-12582912.f, -12582912.f));
  const uint64_t f = f32x2_fma(n, f32x2_pack(-1.f, -1.f), xv);
  uint64_t q = f32x2_fma(f, f32x2_pack(0.055171650f, 0.055171650f),
                         f32x2_pack(0.24261114f, 0.24261114f));
  q = f32x2_fma(q, f, f32x2_pack(0.69326097f, 0.69326097f));
  q = f32x2_fma(q, f, f32x2_pack(0.99992806f, 0.99992806f));
  float t0, t1, q0, q1;
  f32x2_unpack(t, t0, t1);
  f32x2_unpack(q, q0, q1);
  a = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  b = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

constexpr int kPpThreads = 352;
constexpr int kPpStages = 2;
constexpr int kPpHalf = 128 * 128;        // 128 rows x 64 bf16
constexpr int kPpQBytes = 4 * kPpHalf;    // [tile A, B][d half]
constexpr int kPpKVBytes = 4 * kPpHalf;   // K halves, then V halves
constexpr int kPpSmem = kPpQBytes + kPpStages * kPpKVBytes + kBarBytes + 1024;
static_assert(kPpSmem <= 232448, "ping-pong attention: shared memory");

// SPLIT: share of the exponentials of mask-free tiles computed by
// exp2_fma_pair instead of the multi-function unit (0 none, 1 a quarter,
// 2 half of the element pairs).
template <int SPLIT>
__global__ void __launch_bounds__(kPpThreads, 1)
fa_tc_pp_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                const __grid_constant__ CUtensorMap tmv, const FaParams p) {
  constexpr int FD = 128, FN = 128, FNS = kPpStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kPpQBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + FNS * kPpKVBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;            // [FNS]
  uint64_t* k_empty = k_full + FNS;       // [FNS]
  uint64_t* v_full = k_empty + FNS;       // [FNS]
  uint64_t* v_empty = v_full + FNS;       // [FNS]
  uint64_t* s_full = v_empty + FNS;       // [2]: tile A, tile B
  uint64_t* p_full = s_full + 2;          // [2]
  uint64_t* o_done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  unsigned long long* const tl = g_fa_timeline;
  const size_t tl_cta =
      ((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
#define FA_TL(i) \
  do { if (tl) tl[tl_cta * 64 + (i)] = globaltimer(); } while (0)
#define FA_TLJ(j, k) \
  do { if (tl && (j) < 8) tl[tl_cta * 64 + 8 + 7 * (j) + (k)] = globaltimer(); } while (0)
  if (threadIdx.x == 0) FA_TL(0);
  pdl_wait();
  const int seq = blockIdx.y;
  const int kvh = blockIdx.z;
  const int G = p.G;
  const int q0 = p.cu_q[seq];
  const int q_len = p.cu_q[seq + 1] - q0;
  const int seq_len = p.seq_lens[seq];
  const int n_qt = (q_len * G + 2 * FM - 1) / (2 * FM);
  const int qt = (int)gridDim.x - 1 - (int)blockIdx.x;  // longest causal rows first
  if (qt >= n_qt) return;
  const int tpt = FM / G;  // tokens per 128-row tile
  const int t0 = qt * 2 * tpt;
  const int pos_first = seq_len - q_len + t0;
  const int pos_last = seq_len - q_len + min(q_len, t0 + 2 * tpt) - 1;
  int k_lo = p.window > 0 ? max(0, pos_first - p.window + 1) : 0;
  k_lo = (k_lo / FN) * FN;
  const int k_hi = pos_last + 1;
  const int n_tiles = (k_hi - k_lo + FN - 1) / FN;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < FNS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);  // one arrival per softmax warp of the tile
    }
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmq);
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemColsFa);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) {
    pdl_trigger();
    FA_TL(1);
  }
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tS = tmem_base, tO = tmem_base + 2 * FN;  // S_A | S_B | O_A | O_B
  const int BS = p.block_size;
  const int blk_last = (seq_len - 1) >> p.block_shift;

  if (warp == 0 || warp == 6) {
    // ------------------------------------------------- producers (K: 0, V: 6)
    const bool is_v = warp == 6;
    const int* bt = p.block_table + (size_t)seq * p.max_blocks;
    const int nb = FN / BS;
    if (!is_v && lane == 0) {
      mbar_arrive_expect_tx(q_full, (uint32_t)kPpQBytes);
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sQ + (2 * x + h) * kPpHalf, &tmq, q_full, h * 64, kvh * G,
                      q0 + t0 + x * tpt);
    }
    // Cache-block ids are fetched ahead, one warp-wide load per `per` tiles.
    const int per = 32 / nb;
    auto load_ids = [&](int g) -> int {
      const int tile = g * per + lane / nb;
      if (tile >= n_tiles) return 0;
      const int b = ((k_lo + tile * FN) >> p.block_shift) + lane % nb;
      const int id = __ldg(bt + min(b, blk_last));
      return in_bounds(id >= 0 && id < p.num_blocks, p.err) ? id : 0;
    };
    int ids_cur = load_ids(0), ids_next = load_ids(1), g_cur = 0;
    auto issue = [&](int j) -> bool {
      const int g = j / per;
      if (g > g_cur) {
        ids_cur = ids_next;
        ids_next = load_ids(++g_cur + 1);
      }
      const int ids = g == g_cur ? ids_cur : ids_next;
      const int st = j % FNS;
      const uint32_t ph = (uint32_t)((j / FNS) & 1);
      uint64_t* fullb = is_v ? &v_full[st] : &k_full[st];
      int ok = 1;
      if (lane == 0) {
        ok = mbar_wait(is_v ? &v_empty[st] : &k_empty[st], ph ^ 1u, p.err) ? 1 : 0;
        FA_TLJ(j, is_v ? 1 : 0);
        if (ok) mbar_arrive_expect_tx(fullb, (uint32_t)(2 * kPpHalf));
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return false;
      uint8_t* dst = sKV + st * kPpKVBytes + (is_v ? 2 * kPpHalf : 0);
      const CUtensorMap* tm = is_v ? &tmv : &tmk;
      // One (cache block, column half) box per lane, one warp-wide instruction.
      const int bi = lane % nb;
      const int blk = __shfl_sync(0xffffffffu, ids, (j % per) * nb + bi);
      if (lane < 2 * nb) {
        const int h = lane / nb;
        tma_load_3d(dst + h * kPpHalf + bi * BS * 128, tm, fullb, h * 64, kvh * BS, blk);
      }
      return true;
    };
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) ok = issue(j);
    if (!ok) *abort_flag = 1;
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(FM, FN, true);
      constexpr uint32_t idesc_pv = umma_idesc_f16(FM, FD, true) | (1u << 16);  // B MN-major
      bool ok = mbar_wait(q_full, 0, p.err);
      FA_TL(2);
      // S_x = Q_x K^T into S buffer x (commit: s_full[x]).
      auto s_mma = [&](int x, int st) {
        const uint32_t sq = smem_u32(sQ + 2 * x * kPpHalf);
        const uint32_t sk = smem_u32(sKV + st * kPpKVBytes);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint64_t aq = umma_desc_sw128(sq + kb * kPpHalf);
          const uint64_t bk = umma_desc_sw128(sk + kb * kPpHalf);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tS + x * FN, aq + (uint64_t)(2 * k), bk + (uint64_t)(2 * k), idesc_s,
                     (kb > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&s_full[x]);
      };
      // O_x += P_x V with P_x read from the first 64 columns of S buffer x.
      auto pv_mma = [&](int x, int st, bool acc) {
        const uint32_t sv = smem_u32(sKV + st * kPpKVBytes + 2 * kPpHalf);
#pragma unroll
        for (int s = 0; s < FN / 16; ++s) {
          const uint64_t bv = umma_desc_sw128_mn(sv + s * 16 * 128, p.v_lbo, p.v_sbo);
          umma_f16_ts(tO + x * FD, tS + x * FN + s * 8, bv, idesc_pv, (acc || s > 0) ? 1u : 0u);
        }
      };
      if (ok && n_tiles > 0) {
        ok = mbar_wait(&k_full[0], 0, p.err);
        if (ok) {
          tc_fence_after();
          s_mma(0, 0);
          s_mma(1, 0);
          umma_commit(&k_empty[0]);
        }
      }
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j % FNS, nst = (j + 1) % FNS;
        const uint32_t ph = (uint32_t)((j / FNS) & 1), nph = (uint32_t)(((j + 1) / FNS) & 1);
        const bool more = j + 1 < n_tiles;
        // tile A: PV_A(j), then S_A(j + 1) over the consumed P_A(j)
        if (!mbar_wait(&p_full[0], (uint32_t)(j & 1), p.err) ||
            !mbar_wait(&v_full[st], ph, p.err)) {
          ok = false;
          break;
        }
        FA_TLJ(j, 3);
        tc_fence_after();
        pv_mma(0, st, j > 0);
        if (more) {
          if (!mbar_wait(&k_full[nst], nph, p.err)) {
            ok = false;
            break;
          }
          FA_TLJ(j + 1, 2);
          tc_fence_after();
          s_mma(0, nst);
        }
        // tile B: PV_B(j), release V_j, then S_B(j + 1) and release K_{j+1}
        if (!mbar_wait(&p_full[1], (uint32_t)(j & 1), p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        pv_mma(1, st, j > 0);
        umma_commit(&v_empty[st]);
        if (more) {
          s_mma(1, nst);
          umma_commit(&k_empty[nst]);
        }
      }
      if (!ok) *abort_flag = 1;
      umma_commit(o_done);
      mbar_wait(o_done, 0, p.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------- softmax (A: 2-5, B: 7-10)
    const int x = warp >= 7 ? 1 : 0;
    const int q4 = warp & 3;
    const int row = x * FM + q4 * 32 + lane;  // 0..255
    const int stid = (int)threadIdx.x - (x ? 224 : 64);  // 0..127 within the group
    const int t = row / G;
    const int head = kvh * G + row % G;
    const bool valid_row = t0 + t < q_len;
    const int row_pos = seq_len - q_len + t0 + t;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const uint32_t s_row = tS + x * FN + lane_base;
    const uint32_t o_row = tO + x * FD + lane_base;
    // Keys this row may attend to: [key_lo, key_hi] (empty for padding rows).
    const int key_hi = valid_row ? min(row_pos, seq_len - 1) : -1;
    const int key_lo = p.window > 0 ? row_pos - p.window + 1 : 0;
    const float sc = p.scale_log2;
    const uint64_t sc2 = f32x2_pack(sc, sc);
    const bool stamp = x == 0 && stid == 0;
    float m_used = -INFINITY, l = 0.f;  // exponent reference (log2 units) and row sum
    bool ok = true;
    using T_ = std::true_type;
    using F_ = std::false_type;
    for (int j = 0; j < n_tiles; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[x], (uint32_t)(j & 1), p.err));
      if (!ok) break;
      if (stamp && j == 0) FA_TL(3);
      if (stamp) FA_TLJ(j, 4);
      tc_fence_after();
      const int kbase = k_lo + j * FN;
      const int lo = key_lo - kbase, hi = key_hi - kbase;  // in-tile bounds
      const bool masked = __any_sync(0xffffffffu, lo > 0 || hi < FN - 1);
      // Pass 1 over the 128 scores: the row max in log2 units.
      auto row_max = [&](auto masked_c) -> float {
        constexpr bool kMasked = decltype(masked_c)::value;
        float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t r[2][32];
          tmem_ld_32x32b_x32(s_row + h * 64, r[0]);
          tmem_ld_32x32b_x32(s_row + h * 64 + 32, r[1]);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float va = __uint_as_float(r[i >> 4][(2 * i) & 31]);
            float vb = __uint_as_float(r[i >> 4][(2 * i + 1) & 31]);
            if constexpr (kMasked) {
              const int k = h * 64 + 2 * i;
              if (k < lo || k > hi) va = -INFINITY;
              if (k + 1 < lo || k + 1 > hi) vb = -INFINITY;
            }
            mxa = fmaxf(mxa, va);
            mxb = fmaxf(mxb, vb);
          }
        }
        return fmaxf(mxa, mxb) * sc;
      };
      const float mx = masked ? row_max(T_{}) : row_max(F_{});
      // Exponent reference: the first finite max, then lazily the running max
      // whenever a tile's max exceeds it by more than 2^8 (O rescaled then).
      const bool resc = m_used != -INFINITY && mx > m_used + 8.f;
      if (__any_sync(0xffffffffu, resc)) {
        const float alpha = resc ? exp2f(m_used - mx) : 1.f;
        if (resc) {
          l *= alpha;
          m_used = mx;
        }
        if (j > 0) {
          // O_x holds PV_x(j - 1), complete (S_x(j) was committed after it).
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(o_row + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st_32x32b_x32(o_row + c * 32, o);
          }
        }
      }
      if (m_used == -INFINITY) m_used = mx;
      // Pass 2: P = exp2(S * scale - m_used) as bf16 pairs over the first 64
      // columns of this S buffer (half h's P lands in columns half 0 has
      // already read), row sum into l.
      const float mu_eff = m_used == -INFINITY ? 0.f : m_used;
      const uint64_t nmu2 = f32x2_pack(-mu_eff, -mu_eff);
      auto write_p = [&](auto masked_c) -> float {
        constexpr bool kMasked = decltype(masked_c)::value;
        uint64_t acc = f32x2_pack(0.f, 0.f);
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t r[2][32];
          tmem_ld_32x32b_x32(s_row + h * 64, r[0]);
          tmem_ld_32x32b_x32(s_row + h * 64 + 32, r[1]);
          tmem_wait_ld();
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float va = __uint_as_float(r[i >> 4][(2 * i) & 31]);
            float vb = __uint_as_float(r[i >> 4][(2 * i + 1) & 31]);
            if constexpr (kMasked) {
              const int k = h * 64 + 2 * i;
              if (k < lo || k > hi) va = -INFINITY;
              if (k + 1 < lo || k + 1 > hi) vb = -INFINITY;
            }
            float ea, eb;
            f32x2_unpack(f32x2_fma(f32x2_pack(va, vb), sc2, nmu2), ea, eb);
            // (i is a compile-time constant in the unrolled loop)
            if (!kMasked && SPLIT > 0 && (SPLIT == 2 ? (i & 1) == 1 : (i & 3) == 3)) {
              exp2_fma_pair(ea, eb);
            } else {
              ea = fast_exp2(ea);
              eb = fast_exp2(eb);
            }
            acc = f32x2_add(acc, f32x2_pack(ea, eb));
            w[i] = pack_bf16x2(ea, eb);
          }
          tmem_st_32x32b_x32(s_row + h * 32, w);
        }
        float a0, a1;
        f32x2_unpack(acc, a0, a1);
        return a0 + a1;
      };
      l += masked ? write_p(T_{}) : write_p(F_{});
      tmem_wait_st();
      if (x == 0 && j == n_tiles - 1 && kbase + FN > seq_len &&
          __all_sync(0xffffffffu, mbar_wait(&v_full[j % FNS], (uint32_t)((j / FNS) & 1), p.err))) {
        // Zero the V rows past the sequence end (stale cache-block contents)
        // before PV_A of the last tile; PV_B follows PV_A.
        uint8_t* sv = sKV + (j % FNS) * kPpKVBytes + 2 * kPpHalf;
        const int first_bad = max(0, seq_len - kbase);
        for (int idx = stid; idx < (FN - first_bad) * 16; idx += 128) {
          const int key = first_bad + idx / 16, c16 = idx % 16;
          *reinterpret_cast<uint4*>(sv + (c16 >> 3) * kPpHalf + sw_off(key, c16 & 7)) =
              make_uint4(0, 0, 0, 0);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
      }
      // P written, any O correction written: release them to the MMA issuer.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
      if (stamp) FA_TLJ(j, 6);
    }
    if (stamp) FA_TL(4);
    if (!ok) *abort_flag = 1;
    if (ok && n_tiles > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(o_done, 0, p.err));
      if (stamp) FA_TL(5);
      if (ok) {
        tc_fence_after();
        float denom = l;
        if (p.sinks != nullptr) {
          if (m_used == -INFINITY) denom = 1.f;
          else denom += exp2f(p.sinks[head] * 1.4426950408889634f - m_used);
        }
        const float inv = denom > 0.f ? 1.f / denom : 0.f;
        __nv_bfloat16* dst = p.out + (size_t)(q0 + t0 + t) * p.o_stride_t + (size_t)head * FD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(o_row + c * 32, o);  // warp-collective: every lane
          tmem_wait_ld();
          if (valid_row) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[8 * v]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
              w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
              w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
              w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
              *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = w;
            }
          }
        }
      }
    }
  }
  if (threadIdx.x == 64) FA_TL(6);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemColsFa);
  }
  if (threadIdx.x == 0) FA_TL(7);
#undef FA_TL
#undef FA_TLJ
}
