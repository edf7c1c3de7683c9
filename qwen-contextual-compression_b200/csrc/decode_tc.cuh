// Batched decode of 2-8 tokens on the tensor cores (16-bit records, sm_100a).
//
// Included by decode_ffn.cu inside its anonymous namespace: it shares the
// argument structs, the id list handling, the partial-row format and the
// reduce launch of the CUDA-core kernel, and replaces that kernel for 2-8
// tokens, where the per-record dot products (gate and up against every token)
// and their block reductions bind the CUDA-core kernel, not HBM.
//
// Operand layouts (no swizzle, 128-byte core matrices of 8 rows x 16 bytes):
//
// * gate / up: a record's contiguous part r[0..H) read as the K-major no-swizzle
//   operand "8 rows x H/8" -- row i holds r[64b + 8i + kk] for blocks b and
//   kk < 8 (LBO 128 bytes between blocks, SBO = the record's stride) -- so 16
//   records staged one after another form an M = 128 tile with no repacking.
//   The token rows x_t in their natural layout are the matching K-major B
//   operand (N rows (t, i'), x_t[64b + 8i' + kk]).  The MMA then gives
//   D[(r, i), (t, i')] = sum_b,kk r[64b + 8i + kk] x_t[64b + 8i' + kk], and the
//   wanted dot product is its diagonal sum over i = i' (8x the MACs, which the
//   tensor pipe has to spare at N = 8 x tokens).
// * down: y_t[h] = sum_r a[t, r] D_r[h].  A = the down parts as an MN-major
//   no-swizzle operand: MN = (g, m) -> D_r[64g + 8kk + m], K = (r, kk), MN core
//   matrices 128 bytes apart (SBO) and records a stage slot apart (LBO).  B =
//   a block-diagonal expansion of the activations: B[(r, kk), (t, kk')] =
//   a[t, r] if kk = kk' (an 8x8 diagonal block per record and token).  Every
//   entry of D is then an element of y: lane (g, m) of tile j, column (t, kk')
//   holds y_t[1024 j + 64 g + 8 kk' + m].  The activations are split into a
//   16-bit high part and the rounded remainder (two MMAs per step), which keeps
//   a's fp32 precision (the CUDA-core kernel multiplies fp32 a by the weights).
//
// Per CTA (one per SM): a contiguous run of the id list, in groups of 16
// records.  Warp 0 streams each group's records into a ring of 32 KB stages
// with one 2 KB bulk copy per record and stage (its lanes issue them): the
// gate parts in chunks of 1024 elements, then the up parts, then the down
// parts in tiles of 1024 elements.  (A bulk copy costs about 20 ns plus its
// bytes at ~52 GB/s per SM: copies of 1 KB held a stage to ~25 GB/s per SM,
// 2 KB copies reach ~38 GB/s; 16-byte cp.async pieces, alone or beside the
// bulk copies, were slower.)  Warp 1 only joins the block barriers.  Warp 2 holds the
// tensor memory and issues the MMAs (gate and up accumulators of 8 x tokens
// columns, y accumulators of the same width per 1024-element tile), releasing
// each stage with tcgen05.commit.  Warps 3-6 (one per TMEM lane quarter) read the
// gate / up diagonals, apply silu and the token mask, write the diagonal B
// entries, and at the end store the CTA's y as a partial row for the reduce
// launch.  Every wait is bounded; a give-up sets QCC_DEV_TIMEOUT.

constexpr int kTcGroup = 16;         // records per group (M = 128 = 16 records x 8 rows)
constexpr int kTcChunk = 1024;       // gate or up elements per record and stage
constexpr int kTcTile = 1024;        // hidden elements per y tile (M = 128 = 16 x 64)
constexpr int kTcStageBytes = 32768;
constexpr int kTcMaxStages = 6;
constexpr int kTcThreads = 224;      // producer warp, idle warp, MMA warp, four epilogue warps
constexpr int kTcProducers = 64;     // warps 0-1; the x rows are staged by warps 2-6
constexpr int kTcTailFixed = 256;    // mbarriers, TMEM address, give-up flag, counts

struct TcShape {
  int batch;      // tokens (2-8); TP = batch rounded up to even
  int stages;     // ring stages of kTcStageBytes
  int x_off;      // token rows [TP][hidden_pad] (gate|up modes)
  int b_off;      // diagonal B, high then low part, [TP][16 records][64] each (modes with y)
  int tail_off;   // mbarriers etc., then the id cache and token bits
  int tmem_cols;  // allocated TMEM columns (power of two)
  int n_chunks;   // gate stages per group (as many up stages follow)
  int n_tiles;    // down stages per group
};

// Bounded wait that also gives up when another role of the CTA has.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort != 0 || global_timer_ns() - start > kWaitLimitNs) return false;
  }
}

// The same, waited for by lane 0 and broadcast to the warp.
__device__ __forceinline__ bool tc_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort, int lane) {
  bool ok = true;
  if (lane == 0) ok = tc_wait(bar, parity, abort);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// v[O + i] for a lane-dependent i < 8, without local memory.
template <int O>
__device__ __forceinline__ float tc_select8(const float (&v)[16], int i) {
  float r = v[O];
#pragma unroll
  for (int e = 1; e < 8; ++e) r = i == e ? v[O + e] : r;
  return r;
}

template <typename T>
__device__ __forceinline__ T tc_from_f32(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 tc_from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half tc_from_f32<__half>(float v) {
  return __float2half_rn(v);
}

template <typename T, int TP, int MODE>
__global__ void __launch_bounds__(kTcThreads, 1) tc_decode_kernel(const DecodeArgs a, const TcShape L) {
  static_assert(sizeof(T) == 2, "16-bit records only");
  static_assert(TP % 2 == 0 && TP >= 2 && TP <= 8, "N = 8 x TP must be a multiple of 16");
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int N = 8 * TP;
  constexpr bool kGU = MODE != kModeDown;    // gate|up stages and accumulators
  constexpr bool kDN = MODE != kModeGateUp;  // down stages and y accumulators
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int S = L.stages;
  const int seg = a.hidden_pad;
  const int B = L.batch;

  uint8_t* ring = smem;
  T* xs = reinterpret_cast<T*>(smem + L.x_off);
  T* bhi = reinterpret_cast<T*>(smem + L.b_off);
  T* blo = bhi + TP * 1024;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.tail_off);
  uint64_t* empty = full + kTcMaxStages;
  uint64_t* acc_full = empty + kTcMaxStages;  // gate|up accumulators complete (Down: B free again)
  uint64_t* bdown_full = acc_full + 1;        // B written (GateUp: accumulators read), one arrival per epilogue warp
  uint64_t* y_full = acc_full + 2;            // every MMA of the CTA complete
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(acc_full + 4);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  unsigned int* s_count = reinterpret_cast<unsigned int*>(s_tmem + 4);  // [2][kTcThreads / 32]
  int32_t* s_ids = reinterpret_cast<int32_t*>(smem + L.tail_off + kTcTailFixed);
  uint8_t* s_bits = reinterpret_cast<uint8_t*>(s_ids + a.id_cap);

  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (!a.ids_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
  int n = a.n_ids;
  if (a.n_ids_dev != nullptr) n = min(n, max(0, __ldg(a.n_ids_dev)));
  int first = 0;
  const int64_t rebase = a.id_lo >= 0 ? a.id_lo : 0;
  if (a.id_lo >= 0) {
    // The run of an ascending global list inside [id_lo, id_hi), as in the
    // CUDA-core kernel: two counts in one coalesced pass.
    unsigned int below_lo = 0, below_hi = 0;
    for (int i = tid; i < n; i += kTcThreads) {
      const int64_t id = load_id(a, i);
      below_lo += id < a.id_lo ? 1u : 0u;
      below_hi += id < a.id_hi ? 1u : 0u;
    }
    below_lo = __reduce_add_sync(0xffffffffu, below_lo);
    below_hi = __reduce_add_sync(0xffffffffu, below_hi);
    if (lane == 0) {
      s_count[2 * warp] = below_lo;
      s_count[2 * warp + 1] = below_hi;
    }
    __syncthreads();
    unsigned int lo = 0, hi = 0;
    for (int w = 0; w < kTcThreads / 32; ++w) {
      lo += s_count[2 * w];
      hi += s_count[2 * w + 1];
    }
    first = static_cast<int>(lo);
    n = static_cast<int>(hi) - first;
  }
  const int begin = first + static_cast<int>((static_cast<int64_t>(n) * blockIdx.x) / gridDim.x);
  const int end = first + static_cast<int>((static_cast<int64_t>(n) * (blockIdx.x + 1)) / gridDim.x);
  const int cnt = end - begin;
  // With no records (an empty shard) every id is out of range: nothing streams, y is zero.
  const int n_groups = a.n_records > 0 ? (cnt + kTcGroup - 1) / kTcGroup : 0;

  for (int i = tid; i < cnt; i += kTcThreads) {
    const int64_t id = load_id(a, begin + i) - rebase;
    const bool in_range = id >= 0 && id < a.n_records;
    if (!in_range) atomicOr(a.status, QCC_DEV_ID_RANGE);
    s_ids[i] = in_range ? static_cast<int32_t>(id) : -1;
    s_bits[i] = a.token_mask ? static_cast<uint8_t>(__ldg(a.token_mask + begin + i) >> a.mask_shift)
                             : static_cast<uint8_t>(0xFFu);
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(bdown_full, 4);
    mbar_init(y_full, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(s_tmem, static_cast<uint32_t>(L.tmem_cols));
    tmem_relinquish();
  }
  __syncwarp();
  if constexpr (kDN) {
    // Off-diagonal B entries stay zero for the whole launch.
    if (warp >= 3)
      for (int i = tid - 96; i < TP * 2048 * 2 / 16; i += kTcThreads - 96)
        reinterpret_cast<uint4*>(bhi)[i] = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *s_tmem;

  if (warp < 2) {
    // ---------------- producer (warp 0; warp 1 idles): one bulk copy per record and stage ----------------
    const uint64_t policy = policy_evict_first();
    const int64_t part_bytes = static_cast<int64_t>(seg) * 2;
    int s = 0;
    bool ok = true;
    for (int g = 0; g < n_groups && ok && warp == 0; ++g) {
      const int g0 = g * kTcGroup;
      const int rn = min(kTcGroup, cnt - g0);
      const int n_gu = kGU ? 2 * L.n_chunks : 0;
      const int n_st = n_gu + (kDN ? L.n_tiles : 0);
      for (int q = 0; q < n_st; ++q) {
        const int slot = s % S;
        ok = tc_wait_warp(&empty[slot], ((s / S) & 1u) ^ 1u, s_abort, lane);
        if (!ok) break;
        uint8_t* dst = ring + static_cast<size_t>(slot) * kTcStageBytes;
        // Stage q: gate chunk q, up chunk q - n_chunks, or down tile q - n_gu;
        // record r of the group at dst + r * 2 KB.
        int part, bytes, copies;
        int64_t elem;
        if (q < n_gu) {
          part = q < L.n_chunks ? 0 : 1;
          const int c = q - part * L.n_chunks;
          elem = static_cast<int64_t>(c) * kTcChunk;
          bytes = min(kTcChunk, seg - c * kTcChunk) * 2;
          copies = rn;
        } else {
          part = 2;
          const int j = q - n_gu;
          elem = static_cast<int64_t>(j) * kTcTile;
          bytes = min(kTcTile, seg - j * kTcTile) * 2;
          copies = rn + (rn & 1);  // an odd group repeats its last record: both records of an MMA step are finite
        }
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(copies * bytes));
        __syncwarp();
        if (lane < copies) {
          uint8_t* d = dst + lane * (kTcTile * 2);
          const int32_t id = s_ids[g0 + min(lane, rn - 1)];
          // An id outside the records (flagged above) streams record 0; its activation is zero.
          const uint8_t* src = a.packed + static_cast<int64_t>(id >= 0 ? id : 0) * a.record_bytes + part * part_bytes +
                               elem * 2;
          bulk_load(d, src, static_cast<uint32_t>(bytes), &full[slot], policy);
        }
        ++s;
      }
    }
    if (!ok) {
      *s_abort = 1;
      if (lane == 0) atomicOr(a.status, QCC_DEV_TIMEOUT);
    }
    // The copies of the last S issued stages have landed before the CTA exits.
    if (warp == 0 && lane == 0)
      for (int k = max(0, s - S); k < s; ++k) (void)mbar_wait_bounded(&full[k % S], (k / S) & 1u, kWaitLimitNs);
    __syncwarp();
  } else {
    // ---------------- token rows into shared memory (B operand of gate|up) ----------------
    if (a.ids_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
    if constexpr (kGU) {
      const T* xg = reinterpret_cast<const T*>(a.x);
      const int per_row = seg / 8;
      const int total = TP * per_row;
      constexpr int kStride = kTcThreads - kTcProducers;
      // Eight 16-byte loads in flight per thread, then their stores.
      for (int p0 = tid - kTcProducers; p0 < total; p0 += 8 * kStride) {
        uint4 w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int p = p0 + u * kStride;
          const int b = p / per_row;
          const int v = p - b * per_row;
          w[u] = make_uint4(0u, 0u, 0u, 0u);
          if (p < total && b < B) {
            if (a.x_vec) {
              w[u] = __ldg(reinterpret_cast<const uint4*>(xg + b * a.ldx + 8 * v));
            } else {
              __align__(16) T e8[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int h = 8 * v + e;
                e8[e] = h < a.hidden ? xg[b * a.ldx + h] : tc_from_f32<T>(0.f);
              }
              w[u] = *reinterpret_cast<const uint4*>(e8);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int p = p0 + u * kStride;
          if (p < total) reinterpret_cast<uint4*>(xs)[p] = w[u];
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kTcThreads - kTcProducers) : "memory");

    if (warp == 2) {
      // ---------------- MMA issuer ----------------
      if (lane == 0) {
        const uint32_t idesc_gu = idesc_f16_f32(128, N, kBf16, false, false);
        const uint32_t idesc_dn = idesc_f16_f32(128, N, kBf16, true, false);
        const uint32_t ring_a = smem_addr(ring);
        const uint32_t x_a = smem_addr(xs);
        const uint32_t bh_a = smem_addr(bhi);
        const uint32_t bl_a = smem_addr(blo);
        const uint32_t t_gate = tmem;
        const uint32_t t_up = tmem + N;
        const uint32_t t_y = tmem + (kGU ? 2 * N : 0);
        int s = 0;
        bool ok = true;
        for (int g = 0; g < n_groups && ok; ++g) {
          const int rn = min(kTcGroup, cnt - g * kTcGroup);
          if constexpr (MODE == kModeGateUp) {
            if (g > 0) {  // the epilogue has read the previous group's accumulators
              ok = tc_wait(bdown_full, (g - 1) & 1u, s_abort);
              if (!ok) break;
              tc_fence_after_sync();
            }
          }
          if constexpr (kGU) {
            for (int q = 0; q < 2 * L.n_chunks; ++q, ++s) {
              const int slot = s % S;
              ok = tc_wait(&full[slot], (s / S) & 1u, s_abort);
              if (!ok) break;
              tc_fence_after_sync();
              const int c = q < L.n_chunks ? q : q - L.n_chunks;
              const uint32_t t_acc = q < L.n_chunks ? t_gate : t_up;
              const int ks = min(kTcChunk, seg - c * kTcChunk) / 128;
              const uint32_t st = ring_a + slot * kTcStageBytes;
              for (int k = 0; k < ks; ++k) {
                const uint64_t bx = smem_desc_none(x_a + (c * kTcChunk + 128 * k) * 2, 128, seg * 2);
                tc_mma_f16(t_acc, smem_desc_none(st + 256 * k, 128, kTcChunk * 2), bx, idesc_gu,
                           (c > 0 || k > 0) ? 1u : 0u);
              }
              tc_commit(&empty[slot]);
            }
            if (!ok) break;
            tc_commit(acc_full);
          }
          if constexpr (kDN) {
            ok = tc_wait(bdown_full, g & 1u, s_abort);
            if (!ok) break;
            tc_fence_after_sync();
            const int pairs = (rn + 1) / 2;
            for (int j = 0; j < L.n_tiles; ++j, ++s) {
              const int slot = s % S;
              ok = tc_wait(&full[slot], (s / S) & 1u, s_abort);
              if (!ok) break;
              tc_fence_after_sync();
              const uint32_t st = ring_a + slot * kTcStageBytes;
              const uint32_t ty = t_y + j * N;
              for (int p = 0; p < pairs; ++p) {
                const uint64_t ad = smem_desc_none(st + p * 2 * kTcTile * 2, kTcTile * 2, 128);
                tc_mma_f16(ty, ad, smem_desc_none(bh_a + p * 256, 128, 2048), idesc_dn, (g > 0 || p > 0) ? 1u : 0u);
                tc_mma_f16(ty, ad, smem_desc_none(bl_a + p * 256, 128, 2048), idesc_dn, 1u);
              }
              tc_commit(&empty[slot]);
            }
            if (!ok) break;
            if constexpr (MODE == kModeDown) tc_commit(acc_full);  // B may be rewritten
          }
        }
        if (!ok) {
          *s_abort = 1;
          atomicOr(a.status, QCC_DEV_TIMEOUT);
        }
        // Arrives once every MMA issued above has completed (also after a give-up).
        tc_commit(y_full);
        (void)mbar_wait_bounded(y_full, 0, kWaitLimitNs);
      }
      __syncwarp();
    } else {
      // ---------------- epilogue warps 3-6: TMEM lane quarter warp % 4 ----------------
      const int quarter = warp & 3;
      const int row = 32 * quarter + lane;  // M row of the accumulators
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
      const int r = row >> 3;  // record of the group (gate|up rows)
      const int i = row & 7;   // its row / diagonal entry
      bool ok = true;
      for (int g = 0; g < n_groups; ++g) {
        const int li = g * kTcGroup + r;
        const int rn = min(kTcGroup, cnt - g * kTcGroup);
        const int32_t id = r < rn ? s_ids[li] : -1;
        const unsigned bits = r < rn ? s_bits[li] : 0u;
        float act[TP];
        if constexpr (kGU) {
          ok = tc_wait_warp(acc_full, g & 1u, s_abort, lane);
          if (!ok) break;
          tc_fence_after_sync();
          float gs[TP], us[TP];
#pragma unroll
          for (int t2 = 0; t2 < TP; t2 += 2) {
            float v[16];
            tmem_load16(lane_base + 8 * t2, v);
            gs[t2] = tc_select8<0>(v, i);
            gs[t2 + 1] = tc_select8<8>(v, i);
            tmem_load16(lane_base + N + 8 * t2, v);
            us[t2] = tc_select8<0>(v, i);
            us[t2 + 1] = tc_select8<8>(v, i);
          }
          tc_fence_before_sync();
#pragma unroll
          for (int t = 0; t < TP; ++t) {
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) {
              gs[t] += __shfl_xor_sync(0xffffffffu, gs[t], off);
              us[t] += __shfl_xor_sync(0xffffffffu, us[t], off);
            }
            const bool use = id >= 0 && t < B && ((bits >> t) & 1u);
            act[t] = use ? __fdividef(gs[t], 1.f + __expf(-gs[t])) * us[t] : 0.f;
          }
          if constexpr (MODE == kModeGateUp) {
            if (i == 0 && id >= 0) {
#pragma unroll
              for (int t = 0; t < TP; ++t) {
                if (t < B && ((bits >> t) & 1u)) {
                  a.act_out[t * a.ld_act_out + id] = act[t];
                  if (a.score_out != nullptr)
                    a.score_out[t * a.ld_score + id] =
                        a.col_w != nullptr ? fabsf(act[t]) * __ldg(a.col_w + id) : fabsf(act[t]);
                }
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bdown_full);  // accumulators read
            continue;
          }
        } else {
          if (g > 0) {  // the previous group's down MMAs have read B
            ok = tc_wait_warp(acc_full, (g - 1) & 1u, s_abort, lane);
            if (!ok) break;
          }
#pragma unroll
          for (int t = 0; t < TP; ++t) {
            const bool use = id >= 0 && t < B && ((bits >> t) & 1u);
            act[t] = use ? load_as_f32(a.act_in, t * a.ld_act_in + id, a.act_in_dtype) : 0.f;
          }
        }
        if constexpr (kDN) {
#pragma unroll
          for (int t = 0; t < TP; ++t) {
            const T hi = tc_from_f32<T>(act[t]);
            const T lo = tc_from_f32<T>(act[t] - to_f32<T>(hi));
            bhi[t * 1024 + r * 64 + 9 * i] = hi;
            blo[t * 1024 + r * 64 + 9 * i] = lo;
          }
          if (MODE == kModeFull && a.a_out != nullptr && i == 0 && r < rn) {
#pragma unroll
            for (int t = 0; t < TP; ++t)
              if (t < B) store_as(a.a_out, t * a.lda + begin + li, a.a_dtype, act[t]);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(bdown_full);
        }
      }
      if (!ok) {
        *s_abort = 1;
        if (lane == 0) atomicOr(a.status, QCC_DEV_TIMEOUT);
      }
    }
  }

  if constexpr (kDN) {
    // This CTA's y -> its partial row ([B][seg] fp32, slice-major float4
    // columns as the reduce launch reads them), tile by tile through the idle
    // ring: the epilogue warps move the tile from TMEM (lane (g, m) of token
    // t holds y_t[1024 j + 64 g + 8 kk + m], kk < 8) into rows of 1152 floats
    // (8 padding floats after every 64 keep the stores free of bank
    // conflicts), then all warps store it as float4 columns.  A CTA with no
    // records (or a layer with none) stores zeros.
    __syncwarp();
    const bool epi = warp >= 3;
    bool yok = false;
    if (epi) {
      // y is in TMEM only if some group ran (no records: an empty shard).
      yok = n_groups > 0 && tc_wait_warp(y_full, 0, s_abort, lane);
      if (n_groups > 0 && !yok && lane == 0) atomicOr(a.status, QCC_DEV_TIMEOUT);
      tc_fence_after_sync();
    }
    constexpr int kRow = kTcTile + 128;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const int hrow = 64 * (row >> 3) + (row & 7) + 8 * (row >> 3);  // padded position of kk = 0
    const uint32_t t_y = tmem + (kGU ? 2 * N : 0) + (static_cast<uint32_t>(32 * quarter) << 16);
    const int per = a.part_per;
    const float inv_per = 1.f / static_cast<float>(per);
    const int grid = gridDim.x;
    const int nvec = B * seg / 4;
    float* stage = reinterpret_cast<float*>(ring);
    for (int j = 0; j < L.n_tiles; ++j) {
      if (epi) {
        constexpr int kPiece = N % 32 == 0 ? 32 : 16;
#pragma unroll
        for (int c0 = 0; c0 < N; c0 += kPiece) {
          float v[kPiece];
          if (yok) {
            if constexpr (kPiece == 32)
              tmem_load32(t_y + j * N + c0, v);
            else
              tmem_load16(t_y + j * N + c0, v);
          } else {
#pragma unroll
            for (int e = 0; e < kPiece; ++e) v[e] = 0.f;
          }
#pragma unroll
          for (int e = 0; e < kPiece; ++e) {
            const int t = (c0 + e) >> 3;
            const int kk = (c0 + e) & 7;
            if (t < B) stage[t * kRow + hrow + 8 * kk] = v[e];
          }
        }
      }
      asm volatile("bar.sync 2, %0;" ::"r"(kTcThreads) : "memory");
      const int q4 = min(kTcTile, seg - j * kTcTile) / 4;
      for (int w = tid; w < B * q4; w += kTcThreads) {
        const int t = w / q4;
        const int h = 4 * (w - t * q4);
        const float4 val = *reinterpret_cast<const float4*>(stage + t * kRow + h + 8 * (h >> 6));
        const int c = (t * seg + j * kTcTile + h) / 4;
        int blk = __float2int_rz(static_cast<float>(c) * inv_per);
        if (blk * per > c) --blk;
        if ((blk + 1) * per <= c) ++blk;
        const int width = min(per, nvec - blk * per);
        __stcg(a.partials + static_cast<int64_t>(blk) * grid * per + static_cast<int64_t>(blockIdx.x) * width +
                   (c - blk * per),
               val);
      }
      asm volatile("bar.sync 2, %0;" ::"r"(kTcThreads) : "memory");
    }
  }
  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, static_cast<uint32_t>(L.tmem_cols));
  }
}

// Launch shape of the tensor-core kernel for a mode, batch and padded hidden
// size; false when it does not apply (the CUDA-core kernel runs instead).
bool tc_plan(int mode, int batch, int hidden_pad_, int dtype, int max_smem, int id_cap, TcShape* out) {
  if (dtype != QCC_DTYPE_BF16 && dtype != QCC_DTYPE_F16) return false;
  if (batch < 2 || batch > 8 || hidden_pad_ % 128 != 0) return false;
  const bool gu = mode != kModeDown;
  const bool dn = mode != kModeGateUp;
  const int tp = batch + (batch & 1);
  const int n = 8 * tp;
  const int n_chunks = (hidden_pad_ + kTcChunk - 1) / kTcChunk;
  const int n_tiles = (hidden_pad_ + kTcTile - 1) / kTcTile;
  const int cols = (gu ? 2 * n : 0) + (dn ? n_tiles * n : 0);
  if (cols > 512) return false;
  int alloc = 32;
  while (alloc < cols) alloc *= 2;
  const size_t xsize = gu ? static_cast<size_t>(tp) * hidden_pad_ * 2 : 0;
  const size_t bsize = dn ? static_cast<size_t>(2) * tp * 2048 : 0;
  const size_t tail = kTcTailFixed + static_cast<size_t>(id_cap) * 4 + (static_cast<size_t>(id_cap) + 15) / 16 * 16;
  const size_t fixed = xsize + bsize + tail;
  if (static_cast<size_t>(max_smem) <= fixed) return false;
  const int stages = static_cast<int>(std::min<size_t>(kTcMaxStages, (max_smem - fixed) / kTcStageBytes));
  if (stages < 2) return false;
  out->batch = batch;
  out->stages = stages;
  out->x_off = stages * kTcStageBytes;
  out->b_off = out->x_off + static_cast<int>(xsize);
  out->tail_off = out->b_off + static_cast<int>(bsize);
  out->tmem_cols = alloc;
  out->n_chunks = n_chunks;
  out->n_tiles = n_tiles;
  return true;
}

size_t tc_smem_bytes(const TcShape& s, int id_cap) {
  return static_cast<size_t>(s.tail_off) + kTcTailFixed + static_cast<size_t>(id_cap) * 4 +
         (static_cast<size_t>(id_cap) + 15) / 16 * 16;
}

using TcKernelFn = void (*)(const DecodeArgs, const TcShape);

template <typename T, int MODE>
TcKernelFn pick_tc_kernel_tp(int tp) {
  switch (tp) {
    case 2: return tc_decode_kernel<T, 2, MODE>;
    case 4: return tc_decode_kernel<T, 4, MODE>;
    case 6: return tc_decode_kernel<T, 6, MODE>;
    case 8: return tc_decode_kernel<T, 8, MODE>;
    default: return nullptr;
  }
}

template <typename T>
TcKernelFn pick_tc_kernel(int mode, int batch) {
  const int tp = batch + (batch & 1);
  if (mode == kModeGateUp) return pick_tc_kernel_tp<T, kModeGateUp>(tp);
  if (mode == kModeDown) return pick_tc_kernel_tp<T, kModeDown>(tp);
  return pick_tc_kernel_tp<T, kModeFull>(tp);
}
