// extern "C" entry points of libdsv4moe.so (declared in include/dsv4moe.h).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "kernels.cuh"

namespace dsv4 {

// Tuning knobs of the grouped GEMM, read once from the environment:
// DSV4_GEMM_L2PROMO = L2 promotion of the weight tensor maps in bytes (0/64/128/256).
static int env_int(const char* name, int dflt, int lo, int hi) {
  const char* e = getenv(name);
  int v = e ? atoi(e) : dflt;
  return v < lo ? lo : (v > hi ? hi : v);
}
static int gemm_l2promo() {
  static const int v = env_int("DSV4_GEMM_L2PROMO", 256, 0, 256);
  return v;
}

// The library links the CUDA runtime statically, so it keeps its own notion of
// the current device: bind it to the device that owns the caller's buffers.
static void bind_device(const void* dptr) {
  cudaPointerAttributes a;
  if (dptr && cudaPointerGetAttributes(&a, dptr) == cudaSuccess &&
      a.type == cudaMemoryTypeDevice) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != a.device) cudaSetDevice(a.device);
  }
  cudaGetLastError();
}

static int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// ---------------------------------------------------------------------------
// optional stage timing: library-owned CUDA events recorded between the
// kernels of dsv4_moe_forward (also inside stream capture, as graph nodes)
// ---------------------------------------------------------------------------
constexpr int kStageEvents = 7;  // start, gate, plan, permute, gemm1, gemm2, combine
static cudaEvent_t g_stage_ev[kStageEvents];
static bool g_profile = false;

static void stage_mark(int i, cudaStream_t st) {
  if (!g_profile) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  if (cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(g_stage_ev[i], st, cudaEventRecordExternal);
  else
    cudaEventRecord(g_stage_ev[i], st);
}

// Official Gate.forward.  bf16 gate weights over 256 experts run on the
// tensor core: batches of kFusedGateTokens or more with the routing fused
// into the GEMM epilogue, smaller ones as split GEMM partials (when `partials`
// has room for them) summed in a fixed order by the top-k kernel.  Other gates
// use the SIMT logits kernel.  Every path routes bit-exactly on the logits it
// produced.
constexpr int kFusedGateTokens = 2048;

static bool tc_gate_ok(const void* x, const void* w, int w_fp32, int H, int E) {
  return !w_fp32 && E == 256 && H % 64 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(w) & 15) == 0;
}

static long long gate_partials_bytes(int T, int H, int E, int nsm, bool tc, bool allow_fused = true) {
  if (!tc || T <= 0 || (allow_fused && T >= kFusedGateTokens)) return 0;
  int bm, ks;
  gate_gemm_split_shape(T, H, E, nsm, &bm, &ks);
  return (long long)ks * T * E * 4;
}

// Hash-routed layers (hash_table != nullptr) never take the fused path: the
// experts come from the table, so the logits go through partials (or the SIMT
// kernel) and the table lookup happens in the top-k kernel.
static int gate_route(const void* x, const void* w, int w_fp32, const float* bias, int T, int H,
                      int E, int k, float route_scale, float* logits, float* weights,
                      int64_t* indices, float* partials, long long partials_bytes, int nsm,
                      cudaStream_t st, const int64_t* hash_table = nullptr,
                      const int64_t* input_ids = nullptr, long long vocab = 0) {
  const bool hashed = hash_table != nullptr;
  if (tc_gate_ok(x, w, w_fp32, H, E)) {
    const long long need = gate_partials_bytes(T, H, E, nsm, true, !hashed);
    if (need > 0 && partials && partials_bytes >= need) {
      int bm, ks;
      gate_gemm_split_shape(T, H, E, nsm, &bm, &ks);
      int rc = launch_gate_gemm_partials(x, w, T, H, E, partials, nsm, st);
      if (rc) return rc;
      return launch_gate_topk(partials, bias, T, E, k, route_scale, weights, indices, st, ks, logits,
                              hash_table, input_ids, vocab);
    }
    if (!hashed)
      return launch_gate_gemm_topk(x, w, T, H, bias, k, route_scale, logits, weights, indices, nsm, st);
  }
  int rc = launch_gate_logits(x, w, w_fp32, T, H, E, logits, st);
  if (rc) return rc;
  return launch_gate_topk(logits, bias, T, E, k, route_scale, weights, indices, st, 1, nullptr,
                          hash_table, input_ids, vocab);
}

// ---------------------------------------------------------------------------
// workspace layout of one layer call
// ---------------------------------------------------------------------------
struct Plan {
  int T, E, k, H, I, S, block_n, max_rows, max_tiles;
  int split1, split2;  // split-K slices of GEMM1 / GEMM2 (1 = none)
  int part_rows;       // compact rows of the split-K partial sums
  bool fp4;            // routed GEMM1 on FP4 activations (dsv4_set_fp4_activations)
  long long off[25];
  long long total;
};

static long long align256(long long v) { return (v + 255) & ~255LL; }

static int choose_block_n(int T, int k, int E) {
  // tuning override: DSV4_BLOCK_N = 32 | 64 | 128 | 256 (256 = CTA-pair GEMM)
  static const int forced = env_int("DSV4_BLOCK_N", 0, 0, 256);
  if (forced == 32 || forced == 64 || forced == 128 || forced == 256) return forced;
  // rows per routed expert on average; small segments waste less with N = 32.
  // CTA pairs (256-row tiles) only pay where segments are large enough that
  // rounding them to 256 rows costs little: measured on the 8192-token
  // Zipf(1.2) layer (median segment 19 rows), 256-row tiles compute 29% more
  // rows than 128-row tiles and the pair form loses 24% despite being ~5%
  // faster per computed row.
  const long long avg = (long long)T * k / (E > 0 ? E : 1);
  if (avg <= 16 && T <= 256) return 32;
  if (avg <= 48) return 64;
  if (avg <= 2048) return 128;
  return 256;
}

// Split-K slices for the decode-size GEMMs.  With few tokens the layer has few
// (segment tile, weight block) items, each a serial stream of k tiles, and
// 36 of 148 SMs idle at one token; cutting each item's k range into S slices
// (S divides the K/512 scale groups) gives every SM work.  Measured on B200 at
// 1/8/16 tokens the split is no faster than the unsplit GEMM (the per-unit
// accumulator handoff and fixup cost what the idle SMs would have gained), so
// it is off unless asked for: the setting (dsv4_set_k_split; initially
// DSV4_KSPLIT, default 1) is 1 = off, 0 = automatic (>= 16 units per SM,
// slices of at least 8 k tiles), n > 1 = up to n slices.  At most 8 slices
// (the fixup's registers).
static std::atomic<int> g_k_split_setting{-1};

static int k_split_setting() {
  int v = g_k_split_setting.load(std::memory_order_relaxed);
  if (v < 0) {
    v = env_int("DSV4_KSPLIT", 1, 0, 64);
    g_k_split_setting.store(v, std::memory_order_relaxed);
  }
  return v;
}

// FP4 activations for the routed experts' GEMM1 (opt-in: 0 = off, the
// default, matching the reference's e4m3 act_quant; 1 = on).  From
// DSV4_FP4_ACT on first use, or dsv4_set_fp4_activations.
static std::atomic<int> g_fp4_act_setting{-1};
// bumped by every setter: a captured graph records the kernels of the settings
// in force, so callers that cache graphs compare it
static std::atomic<long long> g_settings_generation{0};

static int fp4_act_setting() {
  int v = g_fp4_act_setting.load(std::memory_order_relaxed);
  if (v < 0) {
    v = env_int("DSV4_FP4_ACT", 0, 0, 1);
    g_fp4_act_setting.store(v, std::memory_order_relaxed);
  }
  return v;
}

// The fused decode routing kernel (route_small_fused_kernel) for batches of
// up to 8 tokens: off by default (measured no faster than the three separate
// kernels inside a CUDA graph, slower at 8 tokens); DSV4_FUSED_ROUTE=1 or
// dsv4_set_fused_routing(1) turns it on.
static std::atomic<int> g_fused_route_setting{-1};

static bool small_route_fused_enabled() {
  int v = g_fused_route_setting.load(std::memory_order_relaxed);
  if (v < 0) {
    v = env_int("DSV4_FUSED_ROUTE", 0, 0, 1);
    g_fused_route_setting.store(v, std::memory_order_relaxed);
  }
  return v == 1;
}

static int choose_k_split(int T, int k, int E, int block_n, int nb, int kt, int nsm) {
  const int groups = kt / 4;
  const int setting = k_split_setting();
  if (setting == 1 || block_n > 64 || groups < 2) return 1;
  int s = 1;
  if (setting > 1) {
    while (s * 2 <= setting && s * 2 <= groups && s * 2 <= 8) s *= 2;
  } else {
    const long long tiles = (long long)((long long)T * k < E ? (long long)T * k : E) + 1;
    while (s * 2 <= groups / 2 && s * 2 <= 8 && tiles * nb * s < 16LL * nsm) s *= 2;
  }
  while (groups % s) s >>= 1;
  return s;
}

static int validate(const dsv4_moe_layer* L) {
  if (!L) return DSV4_ERR_ARG;
  // the k-packed activation scale atoms cover four 128-wide k tiles
  if (L->hidden <= 0 || L->inter <= 0 || L->hidden % 512 || L->inter % 512) return DSV4_ERR_ARG;
  if (L->n_routed <= 0 || L->n_routed > 512) return DSV4_ERR_UNSUPPORTED;
  if (L->topk <= 0 || L->topk > 8 || L->topk > L->n_routed) return DSV4_ERR_UNSUPPORTED;
  if (L->n_shared != 0 && L->n_shared != 1) return DSV4_ERR_UNSUPPORTED;
  if (L->gate_w && L->hidden > 8192) return DSV4_ERR_UNSUPPORTED;
  return DSV4_OK;
}

// The CTA-pair GEMM reads scale atoms through 256-byte-row tensor maps: every
// atom buffer must start on 256 bytes and hold whole rows.
static bool pair_layout_ok(const dsv4_moe_layer* L) {
  const long long sc = (long long)L->inter * L->hidden / 32;
  if (sc % 256) return false;
  if (L->arena && ((reinterpret_cast<uintptr_t>(L->arena_sf) & 255) || (L->sf_slot_stride % 256)))
    return false;
  if (L->shared_w1 && (reinterpret_cast<uintptr_t>(L->shared_sf) & 255)) return false;
  return true;
}

// E_local < 0: the whole layer (E = n_routed, gate included); otherwise the
// local experts of an expert-parallel rank (no gate).
static Plan make_plan(const dsv4_moe_layer* L, int T, int E_local = -1) {
  Plan p{};
  p.T = T;
  p.E = E_local < 0 ? L->n_routed : E_local;
  p.k = L->topk;
  p.H = L->hidden;
  p.I = L->inter;
  p.S = L->n_shared;
  p.block_n = choose_block_n(T, p.k, p.E);
  if (p.block_n == 256 && (!pair_layout_ok(L) || pair_clusters_resident(true) <= 0 ||
                           pair_clusters_resident(false) <= 0))
    p.block_n = 128;
  const long long rows = (long long)T * p.k + (long long)T * p.S + 31LL * (p.E + 1);
  p.max_rows = (int)((rows + 31) / 32 * 32);
  p.max_tiles = (int)(((long long)T * p.k + (long long)T * p.S) / p.block_n + p.E + 2);
  const long long atom_groups = p.max_rows / 32 + 4;
  const long long nchunks = T > 0 ? (T + route_chunk_tokens(T) - 1) / route_chunk_tokens(T) : 0;
  const int nsm = num_sms();
  const int nb1 = p.I / 128, nb2 = p.H / 256;
  p.split1 = choose_k_split(T, p.k, p.E, p.block_n, nb1, p.H / 128, nsm);
  p.split2 = choose_k_split(T, p.k, p.E, p.block_n, nb2, p.I / 128, nsm);
  p.part_rows = T * p.k + T * p.S;
  // single-GPU layer only; the CTA-pair form and split-K keep e4m3 activations
  p.fp4 = E_local < 0 && L->arena != nullptr && fp4_act_setting() == 1 && p.block_n != 256 && p.H % 256 == 0 &&
          p.I % 256 == 0;
  if (p.fp4) p.split1 = p.split2 = 1;
  const int smax = p.split1 > p.split2 ? p.split1 : p.split2;
  const long long part_ld = (long long)(nb1 * 256 > nb2 * 256 ? nb1 * 256 : nb2 * 256);
  long long sz[25] = {
      (long long)T * (p.E > p.k ? p.E : p.k) * 4,  // logits (expert parallel: return rows)
      (long long)T * p.k * 4,                 // weights
      (long long)T * p.k * 8,                 // indices
      (long long)(p.E + 1) * 4,               // counts
      (long long)(p.E + 2) * 4,               // seg_start
      16,                                     // n_tiles
      (long long)T * p.k * 4,                 // route_slot
      (long long)p.max_rows * 4,              // slot_token
      (long long)p.max_rows * 4,              // slot_weight
      (long long)p.max_tiles * 16,            // tiles
      (long long)p.max_rows * p.H,            // xq
      atom_groups * (p.H / 512) * 512,        // xsf (k-packed: 4 k tiles per atom)
      (long long)p.max_rows * p.I,            // hq
      atom_groups * (p.I / 512) * 512,        // hsf
      (long long)p.max_rows * p.H * 2,        // O
      E_local < 0 ? gate_partials_bytes(T, p.H, p.E, nsm,
                                        L->gate_w && !L->gate_w_fp32 && p.E == 256)
                  : 0,                        // gate partial logits
      (long long)p.E * nchunks * 4,           // per-chunk expert counts
      (long long)p.E * nchunks * 4,           // per-chunk segment offsets
      16,                                     // plan control words
      smax > 1 ? (long long)smax * p.part_rows * part_ld * 4 : 0,  // split-K partial sums
      smax > 1 ? (long long)p.max_tiles * (nb1 + nb2) * 4 : 0,     // split-K item counters
      p.fp4 ? (long long)p.max_rows * (p.H / 2) : 0,                // FP4 activation codes
      p.fp4 ? atom_groups * (p.H / 128) * 512 : 0,                  // their per-32 scale atoms
      p.fp4 ? (long long)p.max_rows * (p.I / 2) : 0,                // FP4 h codes
      p.fp4 ? atom_groups * (p.I / 128) * 512 : 0,                  // their per-32 scale atoms
  };
  long long o = 0;
  for (int i = 0; i < 25; ++i) {
    p.off[i] = o;
    o += align256(sz[i]);
  }
  p.total = o;
  return p;
}


// Scale-atom maps of the CTA-pair GEMM: routed arena atoms, shared expert
// atoms and the activation atoms `act` (act_bytes), each as 256-byte rows.
// A missing routed or shared part reuses the other's map (never read).
static int make_pair_sf_maps(const dsv4_moe_layer* L, PairMaps* pm, const uint8_t* act,
                             long long act_bytes) {
  const long long sc = (long long)L->inter * L->hidden / 32;
  int rc;
  const bool has_routed = L->arena != nullptr, has_shared = L->shared_w1 != nullptr;
  if (has_routed &&
      (rc = make_tmap_atoms(&pm->sfw, L->arena_sf, (long long)L->n_slots * L->sf_slot_stride, 8)))
    return rc;
  if (has_shared && (rc = make_tmap_atoms(&pm->sfs, L->shared_sf, 3 * sc, 8))) return rc;
  if (!has_routed) pm->sfw = pm->sfs;
  if (!has_shared) pm->sfs = pm->sfw;
  return make_tmap_atoms(&pm->sfx, act, act_bytes, 2);
}

// GEMM1 (w1|w3 + SwiGLU + re-quant) then GEMM2 (w2) over a routing plan.
// out_bf16 receives the expert rows [max_rows, H] (row = plan slot).
// Split-K buffers of one layer call (see choose_k_split); split1/split2 = 1: none.
struct SplitK {
  int split1 = 1, split2 = 1;
  float* partial = nullptr;
  int part_rows = 0;
  int* done1 = nullptr;  // [max_tiles * I/128] GEMM1 item counters
  int* done2 = nullptr;  // [max_tiles * H/256] GEMM2 item counters
};

static SplitK plan_split(const Plan& p, uint8_t* ws) {
  SplitK k;
  if (p.split1 == 1 && p.split2 == 1) return k;
  k.split1 = p.split1;
  k.split2 = p.split2;
  k.partial = reinterpret_cast<float*>(ws + p.off[19]);
  k.part_rows = p.part_rows;
  k.done1 = reinterpret_cast<int*>(ws + p.off[20]);
  k.done2 = k.done1 + (size_t)p.max_tiles * (p.I / 128);
  return k;
}

static int split_counters(const Plan& p) {
  return (p.split1 > 1 || p.split2 > 1) ? p.max_tiles * (p.I / 128 + p.H / 256) : 0;
}

static int run_expert_gemms(const dsv4_moe_layer* L, const int4* tiles, const int* n_tiles,
                            const float* slot_weight, const uint8_t* xq, const uint8_t* xsf,
                            uint8_t* hq, uint8_t* hsf, __nv_bfloat16* out_bf16, int out_ld,
                            int max_rows, int max_tiles, int block_n, const int* expert_slot,
                            int n_routed, int nsm, cudaStream_t st, const SplitK& sk = SplitK(),
                            const uint8_t* xq4 = nullptr, const uint8_t* xsf4 = nullptr,
                            uint8_t* hq4 = nullptr, uint8_t* hsf4 = nullptr) {
  // xq4 != nullptr (FP4-activation mode): the routed experts' rows take FP4
  // activations through both GEMMs (x -> xq4 before GEMM1, h -> hq4 in GEMM1's
  // epilogue); the shared expert's rows keep e4m3 (xq -> hq) on the e4m3 kernel.
  const int H = L->hidden, I = L->inter;
  const bool has_shared = L->shared_w1 != nullptr;
  const bool has_routed = L->arena != nullptr;
  int rc;
  // arena parameter offsets inside a slot (packed order)
  const long long sc = (long long)I * H / 32;
  const long long w1_off = 3 * sc, w2_off = 3 * sc + (long long)I * H / 2,
                  w3_off = 3 * sc + (long long)I * H;
  CUtensorMap a0, a1, s0, s1, b;
  // GEMM1: w1 | w3 over xq
  if (has_routed) {
    if ((rc = make_tmap_fp4_arena(&a0, L->arena + w1_off, H, I, L->n_slots, L->slot_stride, gemm_l2promo())))
      return rc;
    if ((rc = make_tmap_fp4_arena(&a1, L->arena + w3_off, H, I, L->n_slots, L->slot_stride, gemm_l2promo())))
      return rc;
  }
  if (has_shared) {
    if ((rc = make_tmap_u8(&s0, L->shared_w1, H, I, 128))) return rc;
    if ((rc = make_tmap_u8(&s1, L->shared_w3, H, I, 128))) return rc;
  }
  if (!has_routed) {
    a0 = s0;
    a1 = s1;
  }
  if (!has_shared) {
    s0 = a0;
    s1 = a1;
  }
  const bool pair = block_n == 256;
  if ((rc = make_tmap_u8(&b, xq, H, max_rows, pair ? 128 : block_n))) return rc;
  GemmArgs g1{};
  g1.tiles = tiles;
  g1.n_tiles = n_tiles;
  g1.expert_slot = expert_slot;
  g1.n_routed = n_routed;
  g1.kt_count = H / 128;
  g1.nb_count = I / 128;
  g1.sf_routed = L->arena_sf;
  g1.sf_slot_stride = L->sf_slot_stride;
  g1.sf_off0 = 0;
  g1.sf_off1 = sc;
  g1.sf_shared0 = L->shared_sf;
  g1.sf_shared1 = L->shared_sf ? L->shared_sf + sc : nullptr;
  g1.sfb = xsf;
  g1.slot_weight = slot_weight;
  g1.out_q = hq;
  g1.out_sf = hsf;
  g1.out_ld = I;
  g1.swiglu_limit = L->swiglu_limit;
  g1.k_split = pair ? 1 : sk.split1;
  g1.partial = sk.partial;
  g1.part_rows = sk.part_rows;
  g1.part_ld = g1.nb_count * 256;
  g1.item_done = sk.done1;
  // CTA-pair form: maps of the three scale-atom buffers as 256-byte rows
  PairMaps pm;
  int clusters = 0;
  const long long atoms_x = ((long long)max_rows / 32 + 4) * (H / 512) * 512;
  const long long atoms_h = ((long long)max_rows / 32 + 4) * (I / 512) * 512;
  if (pair) {
    clusters = pair_clusters_resident(true);
    if (clusters <= 0) return DSV4_ERR_UNSUPPORTED;
    if ((rc = make_pair_sf_maps(L, &pm, xsf, atoms_x))) return rc;
    pm.w0 = a0;
    pm.w1 = a1;
    pm.s0 = s0;
    pm.s1 = s1;
    pm.x = b;
    const long long work = (long long)max_tiles * g1.nb_count;
    if (work < clusters) clusters = (int)(work > 0 ? work : 1);
    if ((rc = launch_expert_gemm_pair(true, pm, g1, 0, sc >> 8, 0, sc >> 8, clusters, st)))
      return rc;
  } else if (xq4 && has_routed) {
    // FP4 activations: the routed items on kind::mxf4 (packed w1 / w3 maps,
    // 256-wide k tiles, per-32 activation atoms), then the shared expert's
    // items on the e4m3 kernel
    CUtensorMap p0, p1, bx;
    if ((rc = make_tmap_fp4_packed_arena(&p0, L->arena + w1_off, H, I, L->n_slots, L->slot_stride, gemm_l2promo())))
      return rc;
    if ((rc = make_tmap_fp4_packed_arena(&p1, L->arena + w3_off, H, I, L->n_slots, L->slot_stride, gemm_l2promo())))
      return rc;
    if ((rc = make_tmap_u8(&bx, xq4, H / 2, max_rows, block_n))) return rc;
    GemmArgs g4 = g1;
    g4.kt_count = H / 256;
    g4.sfb = xsf4;
    g4.out_q = hq4;
    g4.out_sf = hsf4;
    g4.k_split = 1;
    g4.seg_filter = 1;
    const long long work1 = (long long)max_tiles * g1.nb_count;
    const int grid1 = (int)(work1 < nsm ? work1 : nsm);
    if ((rc = launch_expert_gemm_fp4(true, block_n, p0, p1, bx, g4, grid1, st))) return rc;
    if (has_shared) {
      GemmArgs gs = g1;
      gs.k_split = 1;
      gs.seg_filter = 2;
      if ((rc = launch_expert_gemm(true, block_n, a0, a1, s0, s1, b, gs, grid1, st))) return rc;
    }
  } else {
    const long long work1 = (long long)max_tiles * g1.nb_count * g1.k_split;
    const int grid1 = (int)(work1 < nsm ? work1 : nsm);
    if ((rc = launch_expert_gemm(true, block_n, a0, a1, s0, s1, b, g1, grid1, st))) return rc;
  }
  stage_mark(4, st);

  // GEMM2: w2 over hq
  if (has_routed) {
    if ((rc = make_tmap_fp4_arena(&a0, L->arena + w2_off, I, H, L->n_slots, L->slot_stride, gemm_l2promo())))
      return rc;
  }
  if (has_shared) {
    if ((rc = make_tmap_u8(&s0, L->shared_w2, I, H, 128))) return rc;
  }
  if (!has_routed) a0 = s0;
  if (!has_shared) s0 = a0;
  if ((rc = make_tmap_u8(&b, hq, I, max_rows, pair ? 128 : block_n))) return rc;
  GemmArgs g2 = g1;
  g2.kt_count = I / 128;
  g2.nb_count = H / 256;
  g2.sf_off0 = 2 * sc;
  g2.sf_off1 = 2 * sc;
  g2.sf_shared0 = L->shared_sf ? L->shared_sf + 2 * sc : nullptr;
  g2.sf_shared1 = g2.sf_shared0;
  g2.sfb = hsf;
  g2.out_q = nullptr;
  g2.out_sf = nullptr;
  g2.out_bf16 = out_bf16;
  g2.out_ld = out_ld;
  g2.k_split = pair ? 1 : sk.split2;
  g2.part_ld = g2.nb_count * 256;
  g2.item_done = sk.done2;
  if (pair) {
    int clusters2 = pair_clusters_resident(false);
    if (clusters2 <= 0) return DSV4_ERR_UNSUPPORTED;
    if ((rc = make_pair_sf_maps(L, &pm, hsf, atoms_h))) return rc;
    pm.w0 = a0;
    pm.w1 = a0;
    pm.s0 = s0;
    pm.s1 = s0;
    pm.x = b;
    const long long work = (long long)max_tiles * g2.nb_count;
    if (work < clusters2) clusters2 = (int)(work > 0 ? work : 1);
    rc = launch_expert_gemm_pair(false, pm, g2, (2 * sc) >> 8, (2 * sc) >> 8, (2 * sc) >> 8,
                                 (2 * sc) >> 8, clusters2, st);
  } else if (xq4 && has_routed) {
    // FP4 activations: the routed items on kind::mxf4 over hq4, then the
    // shared expert's items on the e4m3 kernel over hq
    CUtensorMap p2, bh;
    if ((rc = make_tmap_fp4_packed_arena(&p2, L->arena + w2_off, I, H, L->n_slots, L->slot_stride, gemm_l2promo())))
      return rc;
    if ((rc = make_tmap_u8(&bh, hq4, I / 2, max_rows, block_n))) return rc;
    GemmArgs g5 = g2;
    g5.kt_count = I / 256;
    g5.sfb = hsf4;
    g5.k_split = 1;
    g5.seg_filter = 1;
    const long long work2 = (long long)max_tiles * g2.nb_count;
    const int grid2 = (int)(work2 < nsm ? work2 : nsm);
    if ((rc = launch_expert_gemm_fp4(false, block_n, p2, p2, bh, g5, grid2, st))) return rc;
    if (has_shared) {
      GemmArgs gs = g2;
      gs.k_split = 1;
      gs.seg_filter = 2;
      rc = launch_expert_gemm(false, block_n, a0, a0, s0, s0, b, gs, grid2, st);
    }
  } else {
    const long long work2 = (long long)max_tiles * g2.nb_count * g2.k_split;
    const int grid2 = (int)(work2 < nsm ? work2 : nsm);
    rc = launch_expert_gemm(false, block_n, a0, a0, s0, s0, b, g2, grid2, st);
  }
  stage_mark(5, st);
  return rc;
}

// Workspace of one single-expert call: identity plan + activation buffers.
struct ExpertPlan {
  int rows_pad, block_n, max_tiles;
  long long off[8];
  long long total;
};

static ExpertPlan make_expert_plan(const dsv4_moe_layer* L, int T) {
  ExpertPlan p{};
  p.block_n = T <= 32 ? 32 : (T <= 64 ? 64 : 128);
  p.rows_pad = (T + 31) / 32 * 32;
  p.max_tiles = (T + p.block_n - 1) / p.block_n + 1;
  const long long groups = p.rows_pad / 32 + 4;
  long long sz[8] = {
      16,                                        // n_tiles, total_rows
      (long long)p.rows_pad * 4,                 // slot_token
      (long long)p.rows_pad * 4,                 // slot_weight
      (long long)p.max_tiles * 16,               // tiles
      (long long)p.rows_pad * L->hidden,         // xq
      groups * (L->hidden / 512) * 512,          // xsf
      (long long)p.rows_pad * L->inter,          // hq
      groups * (L->inter / 512) * 512,           // hsf
  };
  long long o = 0;
  for (int i = 0; i < 8; ++i) {
    p.off[i] = o;
    o += align256(sz[i]);
  }
  p.total = o;
  return p;
}

}  // namespace dsv4

using namespace dsv4;

extern "C" {

int dsv4_version(void) { return 1; }

int dsv4_set_fused_routing(int on) {
  if (on != 0 && on != 1) return DSV4_ERR_ARG;
  g_fused_route_setting.store(on, std::memory_order_relaxed);
  g_settings_generation.fetch_add(1, std::memory_order_relaxed);
  return DSV4_OK;
}

int dsv4_set_fp4_activations(int on) {
  if (on != 0 && on != 1) return DSV4_ERR_ARG;
  g_fp4_act_setting.store(on, std::memory_order_relaxed);
  g_settings_generation.fetch_add(1, std::memory_order_relaxed);
  return DSV4_OK;
}

int dsv4_fp4_act_quant(const void* x, int M, int K, uint8_t* q, uint8_t* s, void* stream) {
  if (M < 0 || K <= 0 || K % 32) return DSV4_ERR_ARG;
  if (M == 0) return DSV4_OK;
  if (!x || !q || !s || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 15))
    return DSV4_ERR_ARG;
  bind_device(q);
  return launch_fp4_act_quant(x, M, K, q, s, num_sms(), static_cast<cudaStream_t>(stream));
}

int dsv4_set_k_split(int slices) {
  if (slices < 0 || slices > 64) return DSV4_ERR_ARG;
  g_k_split_setting.store(slices, std::memory_order_relaxed);
  g_settings_generation.fetch_add(1, std::memory_order_relaxed);
  return DSV4_OK;
}

long long dsv4_settings_generation(void) { return g_settings_generation.load(std::memory_order_relaxed); }

long long dsv4_kernel_launches(void) { return g_kernel_launches.load(std::memory_order_relaxed); }

const char* dsv4_status_string(int s) {
  switch (s) {
    case DSV4_OK: return "ok";
    case DSV4_ERR_ARG: return "invalid argument";
    case DSV4_ERR_CUDA: return "CUDA error";
    case DSV4_ERR_UNSUPPORTED: return "unsupported shape or option";
    case DSV4_ERR_IO: return "pread failed";
    case DSV4_ERR_SHORT_READ: return "short packed expert read";
    case DSV4_ERR_BOUNDS: return "source slice exceeds storage tensor";
    case DSV4_ERR_SIZE: return "target size does not match expert copy plan";
    case DSV4_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

int dsv4_device_error(int clear, int* code) {
  if (!code) return DSV4_ERR_ARG;
  if (cudaDeviceSynchronize() != cudaSuccess) return DSV4_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dsv4_device_error, sizeof(int)) != cudaSuccess)
    return DSV4_ERR_CUDA;
  *code = v;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_dsv4_device_error, &zero, sizeof(int)) != cudaSuccess)
      return DSV4_ERR_CUDA;
  }
  return DSV4_OK;
}

int dsv4_device_error_async(int* dst, void* stream) {
  if (!dst) return DSV4_ERR_ARG;
  return cudaMemcpyFromSymbolAsync(dst, g_dsv4_device_error, sizeof(int), 0, cudaMemcpyDefault,
                                   static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? DSV4_OK
             : DSV4_ERR_CUDA;
}

int dsv4_profile_enable(int enable) {
  // The events are created once and never destroyed: a CUDA graph captured
  // with profiling on keeps recording them whenever it is replayed, so they
  // must outlive every such graph (disabling only stops new captures and
  // launches from marking stages).
  static bool created = false;
  if (enable && !created) {
    for (int i = 0; i < kStageEvents; ++i)
      if (cudaEventCreate(&g_stage_ev[i]) != cudaSuccess) return DSV4_ERR_CUDA;
    created = true;
  }
  g_profile = enable != 0;
  return DSV4_OK;
}

int dsv4_profile_read(float* stage_ms, int n) {
  if (!g_profile || !stage_ms || n < kStageEvents - 1) return DSV4_ERR_ARG;
  if (cudaEventSynchronize(g_stage_ev[kStageEvents - 1]) != cudaSuccess) return DSV4_ERR_CUDA;
  for (int i = 0; i + 1 < kStageEvents; ++i) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, g_stage_ev[i], g_stage_ev[i + 1]) != cudaSuccess) ms = -1.f;
    stage_ms[i] = ms;
  }
  return DSV4_OK;
}

long long dsv4_moe_workspace_bytes(const dsv4_moe_layer* L, int T) {
  if (validate(L) != DSV4_OK || T < 0) return -1;
  return make_plan(L, T).total;
}

int dsv4_moe_workspace_layout(const dsv4_moe_layer* L, int T, long long* out, int n_out) {
  int rc = validate(L);
  if (rc) return rc;
  if (!out || n_out < 17 || T < 0) return DSV4_ERR_ARG;
  const Plan p = make_plan(L, T);
  for (int i = 0; i < 15; ++i) out[i] = p.off[i];
  out[15] = p.max_rows;
  out[16] = p.block_n;
  if (n_out > 17) out[17] = p.off[15];
  if (n_out > 19) {
    out[18] = p.split1;
    out[19] = p.split2;
  }
  if (n_out > 20) out[20] = p.fp4 ? 1 : 0;
  return DSV4_OK;
}

int dsv4_gate_logits(const void* x, const void* w, int w_is_fp32, int T, int H, int E,
                     float* logits, void* stream) {
  if (!x || !w || !logits || T < 0 || H <= 0 || H % 8 || E <= 0) return DSV4_ERR_ARG;
  if (T == 0) return DSV4_OK;
  if (H > 8192) return DSV4_ERR_UNSUPPORTED;  // gate rows are staged in shared memory
  bind_device(logits);
  return launch_gate_logits(x, w, w_is_fp32, T, H, E, logits, static_cast<cudaStream_t>(stream));
}

int dsv4_gate_topk(const float* logits, const float* bias, int T, int E, int topk,
                   float route_scale, float* weights, int64_t* indices, void* stream) {
  if (!logits || !weights || !indices || T < 0 || E <= 0 || topk <= 0) return DSV4_ERR_ARG;
  if (E > 512 || topk > 8 || topk > E) return DSV4_ERR_UNSUPPORTED;
  bind_device(weights);
  return launch_gate_topk(logits, bias, T, E, topk, route_scale, weights, indices,
                          static_cast<cudaStream_t>(stream));
}

long long dsv4_gate_workspace_bytes(const void* w, int w_is_fp32, int T, int H, int E) {
  if (T < 0 || H <= 0 || E <= 0) return -1;
  return gate_partials_bytes(T, H, E, num_sms(), !w_is_fp32 && E == 256 && H % 64 == 0 && w);
}

int dsv4_gate_route(const void* x, const void* w, int w_is_fp32, const float* bias, int T, int H,
                    int E, int topk, float route_scale, float* logits, float* weights,
                    int64_t* indices, void* workspace, long long workspace_bytes, void* stream) {
  if (!x || !w || !logits || !weights || !indices || T < 0 || H <= 0 || H % 8 || E <= 0 ||
      topk <= 0)
    return DSV4_ERR_ARG;
  if (E > 512 || topk > 8 || topk > E || H > 8192) return DSV4_ERR_UNSUPPORTED;
  if (T == 0) return DSV4_OK;
  bind_device(logits);
  return gate_route(x, w, w_is_fp32, bias, T, H, E, topk, route_scale, logits, weights, indices,
                    static_cast<float*>(workspace), workspace ? workspace_bytes : 0, num_sms(),
                    static_cast<cudaStream_t>(stream));
}

long long dsv4_gate_hash_workspace_bytes(const void* w, int w_is_fp32, int T, int H, int E) {
  if (T < 0 || H <= 0 || E <= 0) return -1;
  return gate_partials_bytes(T, H, E, num_sms(), !w_is_fp32 && E == 256 && H % 64 == 0 && w, false);
}

int dsv4_gate_route_hash(const void* x, const void* w, int w_is_fp32, const int64_t* tid2eid,
                         long long vocab, const int64_t* input_ids, int T, int H, int E, int topk,
                         float route_scale, float* logits, float* weights, int64_t* indices,
                         void* workspace, long long workspace_bytes, void* stream) {
  if (!x || !w || !tid2eid || !input_ids || !logits || !weights || !indices || T < 0 || H <= 0 ||
      H % 8 || E <= 0 || topk <= 0 || vocab <= 0)
    return DSV4_ERR_ARG;
  if (E > 512 || topk > 8 || topk > E || H > 8192) return DSV4_ERR_UNSUPPORTED;
  if (T == 0) return DSV4_OK;
  bind_device(logits);
  return gate_route(x, w, w_is_fp32, nullptr, T, H, E, topk, route_scale, logits, weights, indices,
                    static_cast<float*>(workspace), workspace ? workspace_bytes : 0, num_sms(),
                    static_cast<cudaStream_t>(stream), tid2eid, input_ids, vocab);
}

int dsv4_act_quant(const void* x, int M, int K, uint8_t* q, uint8_t* scale, void* stream) {
  if (!x || !q || !scale || M < 0 || K <= 0 || K % 128) return DSV4_ERR_ARG;
  bind_device(q);
  return launch_act_quant(x, M, K, q, scale, num_sms(), static_cast<cudaStream_t>(stream));
}

int dsv4_moe_forward(const dsv4_moe_layer* L, const void* x, int T, void* y,
                     const float* routing_weights, const int64_t* routing_indices,
                     void* workspace, long long workspace_bytes, void* stream) {
  int rc = validate(L);
  if (rc) return rc;
  if (!x || !y || T < 0 || !L->arena || !L->arena_sf || !L->expert_slot) return DSV4_ERR_ARG;
  if ((routing_weights == nullptr) != (routing_indices == nullptr)) return DSV4_ERR_ARG;
  if (!routing_weights && !L->gate_w) return DSV4_ERR_ARG;
  if (L->n_shared && (!L->shared_w1 || !L->shared_w2 || !L->shared_w3 || !L->shared_sf))
    return DSV4_ERR_ARG;
  if (L->slot_stride % 32 || L->n_slots <= 0) return DSV4_ERR_ARG;
  if (T == 0) return DSV4_OK;
  const Plan p = make_plan(L, T);
  if (!workspace || workspace_bytes < p.total) return DSV4_ERR_WORKSPACE;
  bind_device(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* logits = reinterpret_cast<float*>(ws + p.off[0]);
  float* weights = reinterpret_cast<float*>(ws + p.off[1]);
  int64_t* indices = reinterpret_cast<int64_t*>(ws + p.off[2]);
  int* counts = reinterpret_cast<int*>(ws + p.off[3]);
  int* seg_start = reinterpret_cast<int*>(ws + p.off[4]);
  int* n_tiles = reinterpret_cast<int*>(ws + p.off[5]);
  int* route_slot = reinterpret_cast<int*>(ws + p.off[6]);
  int* slot_token = reinterpret_cast<int*>(ws + p.off[7]);
  float* slot_weight = reinterpret_cast<float*>(ws + p.off[8]);
  int4* tiles = reinterpret_cast<int4*>(ws + p.off[9]);
  uint8_t* xq = ws + p.off[10];
  uint8_t* xsf = ws + p.off[11];
  uint8_t* hq = ws + p.off[12];
  uint8_t* hsf = ws + p.off[13];
  __nv_bfloat16* O = reinterpret_cast<__nv_bfloat16*>(ws + p.off[14]);
  const int nsm = num_sms();
  const int H = p.H, E = p.E, k = p.k;

  const float* rw = routing_weights;
  const int64_t* ri = routing_indices;
  int* chunk_cnt = reinterpret_cast<int*>(ws + p.off[16]);
  int* chunk_base = reinterpret_cast<int*>(ws + p.off[17]);
  int* ctrl = reinterpret_cast<int*>(ws + p.off[18]);
  const SplitK sk = plan_split(p, ws);
  float* partials = reinterpret_cast<float*>(ws + p.off[15]);
  const long long partials_bytes = p.off[16] - p.off[15];
  stage_mark(0, st);
  // decode batches of up to 8 tokens with the tensor-core gate: the gate's
  // split-K partial logits, then top-k + route plan + scatter in one kernel
  const long long fused_need = gate_partials_bytes(T, H, E, nsm, true, true);
  if (!rw && T <= 8 && tc_gate_ok(x, L->gate_w, L->gate_w_fp32, H, E) && fused_need > 0 &&
      partials_bytes >= fused_need && small_route_fused_enabled()) {
    int bm, ks;
    gate_gemm_split_shape(T, H, E, nsm, &bm, &ks);
    if ((rc = launch_gate_gemm_partials(x, L->gate_w, T, H, E, partials, nsm, st))) return rc;
    stage_mark(1, st);
    if ((rc = launch_route_small_fused(partials, ks, logits, L->gate_bias, T, E, k, L->route_scale, weights,
                                       indices, x, H, p.S ? T : 0, p.block_n, p.max_rows, p.max_tiles, chunk_base,
                                       counts, seg_start, tiles, n_tiles, slot_token, slot_weight, ctrl, sk.done1,
                                       split_counters(p), route_slot, xq, xsf, st)))
      return rc;
    rw = weights;
    ri = indices;
    stage_mark(2, st);
  } else {
    if (!rw) {
      if ((rc = gate_route(x, L->gate_w, L->gate_w_fp32, L->gate_bias, T, H, E, k, L->route_scale,
                           logits, weights, indices, partials, partials_bytes, nsm, st)))
        return rc;
      rw = weights;
      ri = indices;
    }
    stage_mark(1, st);
    if ((rc = launch_route_plan(ri, T, k, E, 0, p.S ? T : 0, p.block_n, p.max_rows, p.max_tiles,
                                chunk_cnt, chunk_base, ctrl, counts, seg_start, tiles, n_tiles,
                                slot_token, slot_weight, st, sk.done1, split_counters(p))))
      return rc;
    stage_mark(2, st);
    if ((rc = launch_route_scatter(x, T, nullptr, 0, ri, rw, T, k, E, H, p.S ? T : 0, seg_start,
                                   chunk_base, ctrl, route_slot, slot_token, slot_weight, xq, xsf,
                                   nsm, st)))
      return rc;
  }
  uint8_t* xq4 = p.fp4 ? ws + p.off[21] : nullptr;
  uint8_t* xsf4 = p.fp4 ? ws + p.off[22] : nullptr;
  if (p.fp4 && (rc = launch_fp4_scatter_quant(x, T, H, k, route_slot, p.max_rows, xq4, xsf4, nsm, st)))
    return rc;
  stage_mark(3, st);

  uint8_t* hq4 = p.fp4 ? ws + p.off[23] : nullptr;
  uint8_t* hsf4 = p.fp4 ? ws + p.off[24] : nullptr;
  if ((rc = run_expert_gemms(L, tiles, n_tiles, slot_weight, xq, xsf, hq, hsf, O, H, p.max_rows,
                             p.max_tiles, p.block_n, L->expert_slot, L->n_routed, nsm, st, sk, xq4, xsf4, hq4,
                             hsf4)))
    return rc;
  rc = launch_combine(O, H, route_slot, ri, T, k, p.S ? seg_start + E : nullptr, y, st);
  stage_mark(6, st);
  return rc;
}

long long dsv4_expert_workspace_bytes(const dsv4_moe_layer* L, int T) {
  if (!L || L->hidden % 512 || L->inter % 512 || T < 0) return -1;
  return make_expert_plan(L, T).total;
}

int dsv4_expert_forward(const dsv4_moe_layer* L, int expert, const void* x, int T,
                        const float* row_weights, void* y, void* workspace,
                        long long workspace_bytes, void* stream) {
  if (!L || !x || !y || T < 0 || L->hidden % 512 || L->inter % 512) return DSV4_ERR_ARG;
  if (expert < 0 && (!L->shared_w1 || !L->shared_w2 || !L->shared_w3 || !L->shared_sf))
    return DSV4_ERR_ARG;
  if (expert >= 0 && (!L->arena || !L->arena_sf || !L->expert_slot || expert >= L->n_routed ||
                      L->slot_stride % 32))
    return DSV4_ERR_ARG;
  if (T == 0) return DSV4_OK;
  const ExpertPlan p = make_expert_plan(L, T);
  if (!workspace || workspace_bytes < p.total) return DSV4_ERR_WORKSPACE;
  bind_device(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* n_tiles = reinterpret_cast<int*>(ws + p.off[0]);
  int* total_rows = n_tiles + 1;
  int* slot_token = reinterpret_cast<int*>(ws + p.off[1]);
  float* slot_weight = reinterpret_cast<float*>(ws + p.off[2]);
  int4* tiles = reinterpret_cast<int4*>(ws + p.off[3]);
  uint8_t* xq = ws + p.off[4];
  uint8_t* xsf = ws + p.off[5];
  uint8_t* hq = ws + p.off[6];
  uint8_t* hsf = ws + p.off[7];
  const int nsm = num_sms();
  // the shared expert is segment n_routed; a routed expert keeps its own id
  dsv4_moe_layer Lx = *L;
  int seg = expert;
  if (expert < 0) {
    Lx.arena = nullptr;
    seg = L->n_routed > 0 ? L->n_routed : 0;
    Lx.n_routed = seg;
  } else {
    Lx.shared_w1 = Lx.shared_w2 = Lx.shared_w3 = nullptr;
    Lx.shared_sf = nullptr;
  }
  int rc;
  if ((rc = launch_single_segment_plan(T, seg, p.block_n, p.rows_pad, row_weights, slot_token,
                                       slot_weight, tiles, n_tiles, total_rows, st)))
    return rc;
  if ((rc = launch_permute_quant(x, L->hidden, slot_token, total_rows, p.rows_pad, xq, xsf, nsm,
                                 st)))
    return rc;
  // rows are tokens and the epilogue stores only rows < T, so GEMM2 writes y
  return run_expert_gemms(&Lx, tiles, n_tiles, slot_weight, xq, xsf, hq, hsf,
                          static_cast<__nv_bfloat16*>(y), L->hidden, p.rows_pad, p.max_tiles,
                          p.block_n, L->expert_slot, Lx.n_routed, nsm, st);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Dense FP8 linear layers (the attention block's projections): act_quant of x
// then the non-gated grouped GEMM over one segment of M rows, B = the e4m3
// weight with its 128x128 block scales expanded into scale atoms.
// ---------------------------------------------------------------------------
namespace dsv4 {

struct LinearPlan {
  int rows_pad, block_n, max_tiles, split;
  long long off[8];
  long long total;
};

// A linear layer of few rows has few work items (one per 256 output features
// and row tile): N = 1024 at decode is 4 items for 148 SMs.  Under the split-K
// setting (dsv4_set_k_split: 1 = off, the default; 0 = auto; n = up to n) its
// k range is cut into S slices of whole scale groups: in auto, the largest
// power of two up to 8 that divides the groups and keeps items x S within the
// SM count.
static int linear_split(int tiles, int N, int K, int block_n, int nsm) {
  const int groups = K / 512;
  const int setting = k_split_setting();
  if (setting == 1 || block_n > 64) return 1;
  const long long work = (long long)tiles * (N / 256);
  const int cap = setting > 1 ? (setting < 8 ? setting : 8) : 8;
  int s = 1;
  while (s * 2 <= cap && groups % (s * 2) == 0 && (setting > 1 || work * s * 2 <= nsm)) s *= 2;
  return s;
}

static LinearPlan make_linear_plan(int M, int N, int K) {
  LinearPlan p{};
  p.block_n = M <= 32 ? 32 : (M <= 64 ? 64 : 128);
  p.rows_pad = (M + 31) / 32 * 32;
  p.max_tiles = (M + p.block_n - 1) / p.block_n + 1;
  p.split = linear_split((M + p.block_n - 1) / p.block_n, N, K, p.block_n, num_sms());
  const long long groups = p.rows_pad / 32 + 4;
  long long sz[8] = {
      16,                                  // n_tiles, total_rows
      (long long)p.rows_pad * 4,           // slot_token
      (long long)p.rows_pad * 4,           // slot_weight (unused by the non-gated epilogue)
      (long long)p.max_tiles * 16,         // tiles
      (long long)p.rows_pad * K,           // xq
      groups * (K / 512) * 512,            // xsf
      p.split > 1 ? (long long)p.split * p.rows_pad * N * 4 : 0,     // split-K partial sums
      p.split > 1 ? (long long)p.max_tiles * (N / 256) * 4 : 0,      // split-K item counters
  };
  long long o = 0;
  for (int i = 0; i < 8; ++i) {
    p.off[i] = o;
    o += align256(sz[i]);
  }
  p.total = o;
  return p;
}

static bool linear_shape_ok(int M, int N, int K) { return M >= 0 && N > 0 && K > 0 && N % 256 == 0 && K % 512 == 0; }

}  // namespace dsv4

extern "C" {

long long dsv4_fp8_weight_atoms_bytes(int N, int K) {
  if (N <= 0 || K <= 0 || N % 128 || K % 128) return -1;
  return (long long)N * K / 32;
}

int dsv4_build_fp8_weight_atoms(const uint8_t* scale, int N, int K, uint8_t* atoms, void* stream) {
  if (!scale || !atoms || N <= 0 || K <= 0 || N % 128 || K % 128) return DSV4_ERR_ARG;
  bind_device(atoms);
  return launch_build_sf_fp8(scale, N, K, atoms, num_sms(), static_cast<cudaStream_t>(stream));
}

long long dsv4_fp8_linear_workspace_bytes(int M, int N, int K) {
  if (!linear_shape_ok(M, N, K)) return -1;
  return make_linear_plan(M, N, K).total;
}

int dsv4_fp8_linear(const void* x, int M, int K, const uint8_t* w, const uint8_t* w_atoms, int N, void* y,
                    void* workspace, long long workspace_bytes, void* stream) {
  if (!linear_shape_ok(M, N, K)) return N % 256 || K % 512 ? DSV4_ERR_UNSUPPORTED : DSV4_ERR_ARG;
  if (M == 0) return DSV4_OK;
  if (!x || !w || !w_atoms || !y) return DSV4_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(y) & 15))
    return DSV4_ERR_ARG;
  const LinearPlan p = make_linear_plan(M, N, K);
  if (!workspace || workspace_bytes < p.total) return DSV4_ERR_WORKSPACE;
  bind_device(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* n_tiles = reinterpret_cast<int*>(ws + p.off[0]);
  int* total_rows = n_tiles + 1;
  int* slot_token = reinterpret_cast<int*>(ws + p.off[1]);
  float* slot_weight = reinterpret_cast<float*>(ws + p.off[2]);
  int4* tiles = reinterpret_cast<int4*>(ws + p.off[3]);
  uint8_t* xq = ws + p.off[4];
  uint8_t* xsf = ws + p.off[5];
  const int nsm = num_sms();
  int rc;
  // one segment (id 0 with no routed experts: the e4m3 "shared" weight path)
  if ((rc = launch_single_segment_plan(M, 0, p.block_n, p.rows_pad, nullptr, slot_token, slot_weight, tiles,
                                       n_tiles, total_rows, st)))
    return rc;
  if ((rc = launch_permute_quant(x, K, slot_token, total_rows, p.rows_pad, xq, xsf, nsm, st))) return rc;
  CUtensorMap tw, tx;
  if ((rc = make_tmap_u8(&tw, w, K, N, 128))) return rc;
  if ((rc = make_tmap_u8(&tx, xq, K, p.rows_pad, p.block_n))) return rc;
  GemmArgs g{};
  g.tiles = tiles;
  g.n_tiles = n_tiles;
  g.n_routed = 0;
  g.kt_count = K / 128;
  g.nb_count = N / 256;
  g.sf_shared0 = w_atoms;
  g.sf_shared1 = w_atoms;
  g.sfb = xsf;
  g.slot_weight = slot_weight;
  g.out_bf16 = static_cast<__nv_bfloat16*>(y);
  g.out_ld = N;
  g.k_split = p.split;
  if (p.split > 1) {
    g.partial = reinterpret_cast<float*>(ws + p.off[6]);
    g.part_rows = p.rows_pad;
    g.part_ld = N;
    g.item_done = reinterpret_cast<int*>(ws + p.off[7]);
    if (cudaMemsetAsync(g.item_done, 0, (size_t)p.max_tiles * g.nb_count * 4, st) != cudaSuccess)
      return DSV4_ERR_CUDA;
  }
  const long long work = (long long)p.max_tiles * g.nb_count * p.split;
  const int grid = (int)(work < nsm ? work : nsm);
  return launch_expert_gemm(false, p.block_n, tw, tw, tw, tw, tx, g, grid, st);
}

long long dsv4_sparse_attn_workspace_bytes(int B, int S, int K) {
  if (B < 0 || S < 0 || K <= 0) return -1;
  return sparse_attn_workspace(B * S, K, num_sms(), nullptr, nullptr);
}

int dsv4_sparse_attn(const void* q, const void* kv, const float* attn_sink, const int* topk_idxs, int B, int S,
                     int H, int N, int D, int K, float softmax_scale, void* out, void* workspace,
                     long long workspace_bytes, void* stream) {
  if (B < 0 || S < 0 || N <= 0 || K <= 0) return DSV4_ERR_ARG;
  if (H != 64 || D != 512) return DSV4_ERR_UNSUPPORTED;
  if ((long long)B * S == 0) return DSV4_OK;
  if (!q || !kv || !attn_sink || !topk_idxs || !out) return DSV4_ERR_ARG;
  // 16-byte row copies in, 2-byte stores out
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(kv) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 3))
    return DSV4_ERR_ARG;
  bind_device(out);
  return launch_sparse_attn(q, kv, attn_sink, topk_idxs, B, S, N, K, softmax_scale, out, workspace,
                            workspace ? workspace_bytes : 0, num_sms(), static_cast<cudaStream_t>(stream));
}

int dsv4_materialize(const uint8_t* slab, const long long* src_off, const int* dst_slot, int n,
                     int hidden, int inter, uint8_t* arena, long long slot_stride,
                     uint8_t* arena_sf, long long sf_slot_stride, void* bf16_out,
                     long long bf16_slot_stride, void* stream) {
  if (!slab || !src_off || !dst_slot || n < 0 || hidden % 128 || inter % 128) return DSV4_ERR_ARG;
  const long long block = 3LL * inter * hidden / 32 + 3LL * inter * hidden / 2;
  if (arena && slot_stride < block) return DSV4_ERR_ARG;
  if (arena_sf && sf_slot_stride < 3LL * inter * hidden / 32) return DSV4_ERR_ARG;
  if (arena && slot_stride % 16) return DSV4_ERR_ARG;
  // 16-byte vector loads and stores throughout
  if ((reinterpret_cast<uintptr_t>(slab) & 15) || (reinterpret_cast<uintptr_t>(arena) & 15) ||
      (reinterpret_cast<uintptr_t>(bf16_out) & 15) || (bf16_out && bf16_slot_stride % 8))
    return DSV4_ERR_ARG;
  bind_device(slab);
  return launch_materialize(slab, src_off, dst_slot, n, block, arena, slot_stride, hidden, inter,
                            arena_sf, sf_slot_stride, bf16_out, bf16_slot_stride, num_sms(),
                            static_cast<cudaStream_t>(stream));
}

int dsv4_build_scale_atoms(const uint8_t* arena, long long slot_stride, const int* slots, int n,
                           int hidden, int inter, uint8_t* arena_sf, long long sf_slot_stride,
                           void* stream) {
  if (!arena || !slots || !arena_sf || n < 0 || hidden % 128 || inter % 128) return DSV4_ERR_ARG;
  if (sf_slot_stride < 3LL * inter * hidden / 32) return DSV4_ERR_ARG;
  bind_device(arena);
  return launch_build_sf_fp4_arena(arena, slot_stride, slots, n, hidden, inter, arena_sf,
                                   sf_slot_stride, num_sms(), static_cast<cudaStream_t>(stream));
}

int dsv4_build_shared_scale_atoms(const uint8_t* w1_scale, const uint8_t* w2_scale,
                                  const uint8_t* w3_scale, int hidden, int inter,
                                  uint8_t* shared_sf, void* stream) {
  if (!w1_scale || !w2_scale || !w3_scale || !shared_sf || hidden % 128 || inter % 128)
    return DSV4_ERR_ARG;
  bind_device(shared_sf);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long sc = (long long)inter * hidden / 32;
  const int nsm = num_sms();
  int rc;
  if ((rc = launch_build_sf_fp8(w1_scale, inter, hidden, shared_sf, nsm, st))) return rc;
  if ((rc = launch_build_sf_fp8(w3_scale, inter, hidden, shared_sf + sc, nsm, st))) return rc;
  return launch_build_sf_fp8(w2_scale, hidden, inter, shared_sf + 2 * sc, nsm, st);
}

// ---------------------------------------------------------------------------
// expert parallelism (ep.cu): dispatch, owning-rank forward, combine
// ---------------------------------------------------------------------------
static int ep_check(const dsv4_moe_layer* L, int rank, int world) {
  int rc = validate(L);
  if (rc) return rc;
  if (world < 1 || world > 8 || rank < 0 || rank >= world) return DSV4_ERR_ARG;
  if (L->n_routed % world) return DSV4_ERR_ARG;
  return DSV4_OK;
}

long long dsv4_ep_row_bytes(int hidden, int topk) {
  if (hidden <= 0 || hidden % 512 || topk <= 0 || topk > 8) return -1;
  return ep_row_bytes(hidden, topk);
}

long long dsv4_ep_dispatch_workspace_bytes(int T, int world) {
  if (T < 0 || world < 1 || world > 8) return -1;
  return ep_dispatch_workspace(T, world);
}

int dsv4_ep_dispatch(const void* x, const int64_t* indices, const float* weights, int T,
                     int hidden, int topk, int n_routed, int world, void* send,
                     long long send_rows, int* send_counts, int* ret_pos, void* workspace,
                     long long workspace_bytes, void* stream) {
  if (T < 0 || hidden <= 0 || hidden % 512 || topk <= 0 || topk > 8 || world < 1 || world > 8 ||
      n_routed <= 0 || n_routed > 512 || n_routed % world || topk > n_routed || !send_counts)
    return DSV4_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bind_device(send_counts);
  if (T == 0) return cudaMemsetAsync(send_counts, 0, 2 * world * sizeof(int), st) == cudaSuccess
                         ? DSV4_OK : DSV4_ERR_CUDA;
  if (!x || !indices || !weights || !send || !ret_pos) return DSV4_ERR_ARG;
  if (send_rows < (long long)T * (world < topk ? world : topk)) return DSV4_ERR_WORKSPACE;
  if (!workspace || workspace_bytes < ep_dispatch_workspace(T, world)) return DSV4_ERR_WORKSPACE;
  return launch_ep_dispatch(x, indices, weights, T, hidden, topk, n_routed, world,
                            static_cast<uint8_t*>(send), send_counts, ret_pos,
                            static_cast<uint8_t*>(workspace), num_sms(), st);
}

long long dsv4_ep_expert_workspace_bytes(const dsv4_moe_layer* L, int world, int T_own, int R) {
  if (ep_check(L, 0, world) || T_own < 0 || R < 0) return -1;
  return make_plan(L, T_own + R, L->n_routed / world).total;
}

int dsv4_ep_expert_forward(const dsv4_moe_layer* L, int rank, int world, const void* x_own,
                           int T_own, const void* recv, int R, const int* recv_counts,
                           void* ret_send, long long ret_rows, void* workspace,
                           long long workspace_bytes, void* stream) {
  int rc = ep_check(L, rank, world);
  if (rc) return rc;
  if (T_own < 0 || R < 0 || (T_own && !x_own) || (R && (!recv || !recv_counts || !ret_send)) ||
      ret_rows < 0)
    return DSV4_ERR_ARG;
  if (!L->arena || !L->arena_sf || !L->expert_slot || L->slot_stride % 32 || L->n_slots <= 0)
    return DSV4_ERR_ARG;
  if (L->n_shared && (!L->shared_w1 || !L->shared_w2 || !L->shared_w3 || !L->shared_sf))
    return DSV4_ERR_ARG;
  const int T = T_own + R;
  if (T == 0) return DSV4_OK;
  const int e_count = L->n_routed / world, e_begin = rank * e_count;
  const Plan p = make_plan(L, T, e_count);
  if (!workspace || workspace_bytes < p.total) return DSV4_ERR_WORKSPACE;
  bind_device(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* ret_dst = reinterpret_cast<int*>(ws + p.off[0]);
  float* w_local = reinterpret_cast<float*>(ws + p.off[1]);
  int64_t* idx_local = reinterpret_cast<int64_t*>(ws + p.off[2]);
  int* counts = reinterpret_cast<int*>(ws + p.off[3]);
  int* seg_start = reinterpret_cast<int*>(ws + p.off[4]);
  int* n_tiles = reinterpret_cast<int*>(ws + p.off[5]);
  int* route_slot = reinterpret_cast<int*>(ws + p.off[6]);
  int* slot_token = reinterpret_cast<int*>(ws + p.off[7]);
  float* slot_weight = reinterpret_cast<float*>(ws + p.off[8]);
  int4* tiles = reinterpret_cast<int4*>(ws + p.off[9]);
  uint8_t* xq = ws + p.off[10];
  uint8_t* xsf = ws + p.off[11];
  uint8_t* hq = ws + p.off[12];
  uint8_t* hsf = ws + p.off[13];
  __nv_bfloat16* O = reinterpret_cast<__nv_bfloat16*>(ws + p.off[14]);
  int* chunk_cnt = reinterpret_cast<int*>(ws + p.off[16]);
  int* chunk_base = reinterpret_cast<int*>(ws + p.off[17]);
  int* ctrl = reinterpret_cast<int*>(ws + p.off[18]);
  const int nsm = num_sms();
  const int H = p.H, k = p.k;
  const int shared_rows = p.S ? T_own : 0;
  const uint8_t* rows_in = static_cast<const uint8_t*>(recv);
  // profile stages here: unpack, plan, scatter, GEMM1, GEMM2, return gather
  stage_mark(0, st);
  if ((rc = launch_ep_unpack(rows_in, R, T_own, k, H, e_begin, e_count, recv_counts, world,
                             idx_local, w_local, ret_dst, st)))
    return rc;
  stage_mark(1, st);
  const SplitK sk = plan_split(p, ws);
  if ((rc = launch_route_plan(idx_local, T, k, e_count, 1, shared_rows, p.block_n, p.max_rows,
                              p.max_tiles, chunk_cnt, chunk_base, ctrl, counts, seg_start, tiles,
                              n_tiles, slot_token, slot_weight, st, sk.done1, split_counters(p))))
    return rc;
  stage_mark(2, st);
  if ((rc = launch_route_scatter(x_own, T_own, rows_in, ep_row_bytes(H, k), idx_local, w_local, T,
                                 k, e_count, H, shared_rows, seg_start, chunk_base, ctrl,
                                 route_slot, slot_token, slot_weight, xq, xsf, nsm, st)))
    return rc;
  stage_mark(3, st);
  if ((rc = run_expert_gemms(L, tiles, n_tiles, slot_weight, xq, xsf, hq, hsf, O, H, p.max_rows,
                             p.max_tiles, p.block_n, L->expert_slot + e_begin, e_count, nsm, st, sk)))
    return rc;
  rc = launch_ep_return_gather(O, H, route_slot, ret_dst, T * k, ret_rows, ret_send, nsm, st);
  stage_mark(6, st);
  return rc;
}

// ---------------------------------------------------------------------------
// expert parallelism over peer memory (NVLink P2P stores, bounded flag waits)
// ---------------------------------------------------------------------------
long long dsv4_ep_exchange_bytes(int hidden, int topk, int world, int cap_tokens) {
  if (hidden <= 0 || hidden % 512 || topk <= 0 || topk > 8 || world <= 0 || world > 8 ||
      cap_tokens <= 0 || (long long)cap_tokens * topk >= (1 << 24))
    return -1;
  return ep_exchange_bytes(hidden, topk, world, cap_tokens);
}

int dsv4_ep_exchange_alloc(int device, long long bytes, void** out) {
  if (!out || bytes <= 0 || device < 0) return DSV4_ERR_ARG;
  *out = nullptr;
  if (cudaSetDevice(device) != cudaSuccess) return DSV4_ERR_CUDA;
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) {
    cudaGetLastError();
    return DSV4_ERR_CUDA;
  }
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess) {
    cudaFree(p);
    return DSV4_ERR_CUDA;
  }
  *out = p;
  return DSV4_OK;
}

int dsv4_ep_exchange_free(void* p) {
  if (!p) return DSV4_OK;
  bind_device(p);
  return cudaFree(p) == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

int dsv4_ipc_handle(const void* p, uint8_t* handle) {
  if (!p || !handle) return DSV4_ERR_ARG;
  bind_device(p);
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(p)) != cudaSuccess) {
    cudaGetLastError();
    return DSV4_ERR_CUDA;
  }
  static_assert(sizeof(h) == DSV4_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return DSV4_OK;
}

int dsv4_ipc_open(int device, const uint8_t* handle, void** out) {
  if (!handle || !out || device < 0) return DSV4_ERR_ARG;
  *out = nullptr;
  if (cudaSetDevice(device) != cudaSuccess) return DSV4_ERR_CUDA;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return DSV4_ERR_CUDA;
  }
  *out = p;
  return DSV4_OK;
}

int dsv4_ipc_close(void* p) {
  if (!p) return DSV4_OK;
  return cudaIpcCloseMemHandle(p) == cudaSuccess ? DSV4_OK : DSV4_ERR_CUDA;
}

long long dsv4_ep_p2p_dispatch_workspace_bytes(int T, int world) {
  if (T < 0 || world <= 0 || world > 8) return -1;
  return ep_dispatch_workspace(T, world) + 256;
}

int dsv4_ep_dispatch_p2p(const void* x, const int64_t* indices, const float* weights, int T,
                         int hidden, int topk, int n_routed, int world, int rank,
                         const uint64_t* peer_bases, int cap_tokens, int epoch, int* ret_pos,
                         void* workspace, long long workspace_bytes, void* stream) {
  if (world <= 0 || world > 8 || rank < 0 || rank >= world || n_routed % world || hidden % 512 ||
      topk <= 0 || topk > 8 || !peer_bases || cap_tokens <= 0 || T < 0 || T > cap_tokens)
    return DSV4_ERR_ARG;
  if (T && (!x || !indices || !weights || !ret_pos)) return DSV4_ERR_ARG;
  const long long need = ep_dispatch_workspace(T, world) + 256;
  if (!workspace || workspace_bytes < need) return DSV4_ERR_WORKSPACE;
  bind_device(workspace);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* send_counts = reinterpret_cast<int*>(ws + ep_dispatch_workspace(T, world));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0)  // no rows, but every owner still learns that nothing comes from this rank
    return launch_ep_signal_empty(peer_bases, rank, world, send_counts, ws, epoch, st);
  return launch_ep_dispatch(x, indices, weights, T, hidden, topk, n_routed, world, nullptr,
                            send_counts, ret_pos, ws, num_sms(), st, peer_bases, rank, cap_tokens,
                            epoch);
}

long long dsv4_ep_p2p_expert_workspace_bytes(const dsv4_moe_layer* L, int world, int T_own,
                                             int cap_tokens) {
  if (ep_check(L, 0, world) || T_own < 0 || cap_tokens <= 0) return -1;
  return make_plan(L, T_own + world * cap_tokens, L->n_routed / world).total;
}

int dsv4_ep_expert_forward_p2p(const dsv4_moe_layer* L, int rank, int world, const void* x_own,
                               int T_own, void* exchange, const uint64_t* peer_bases,
                               int cap_tokens, int epoch, void* workspace,
                               long long workspace_bytes, void* stream) {
  int rc = ep_check(L, rank, world);
  if (rc) return rc;
  if (T_own < 0 || T_own > cap_tokens || (T_own && !x_own) || !exchange || !peer_bases ||
      cap_tokens <= 0)
    return DSV4_ERR_ARG;
  if (!L->arena || !L->arena_sf || !L->expert_slot || L->slot_stride % 32 || L->n_slots <= 0)
    return DSV4_ERR_ARG;
  if (L->n_shared && (!L->shared_w1 || !L->shared_w2 || !L->shared_w3 || !L->shared_sf))
    return DSV4_ERR_ARG;
  const int T = T_own + world * cap_tokens;
  const int e_count = L->n_routed / world, e_begin = rank * e_count;
  const Plan p = make_plan(L, T, e_count);
  if (!workspace || workspace_bytes < p.total) return DSV4_ERR_WORKSPACE;
  bind_device(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* ret_dst = reinterpret_cast<int*>(ws + p.off[0]);
  float* w_local = reinterpret_cast<float*>(ws + p.off[1]);
  int64_t* idx_local = reinterpret_cast<int64_t*>(ws + p.off[2]);
  int* counts = reinterpret_cast<int*>(ws + p.off[3]);
  int* seg_start = reinterpret_cast<int*>(ws + p.off[4]);
  int* n_tiles = reinterpret_cast<int*>(ws + p.off[5]);
  int* route_slot = reinterpret_cast<int*>(ws + p.off[6]);
  int* slot_token = reinterpret_cast<int*>(ws + p.off[7]);
  float* slot_weight = reinterpret_cast<float*>(ws + p.off[8]);
  int4* tiles = reinterpret_cast<int4*>(ws + p.off[9]);
  uint8_t* xq = ws + p.off[10];
  uint8_t* xsf = ws + p.off[11];
  uint8_t* hq = ws + p.off[12];
  uint8_t* hsf = ws + p.off[13];
  __nv_bfloat16* O = reinterpret_cast<__nv_bfloat16*>(ws + p.off[14]);
  int* chunk_cnt = reinterpret_cast<int*>(ws + p.off[16]);
  int* chunk_base = reinterpret_cast<int*>(ws + p.off[17]);
  int* ctrl = reinterpret_cast<int*>(ws + p.off[18]);
  const int nsm = num_sms();
  const int H = p.H, k = p.k;
  const int shared_rows = p.S ? T_own : 0;
  uint8_t* exch = static_cast<uint8_t*>(exchange);
  stage_mark(0, st);
  // every source's rows and counts are in place
  if ((rc = launch_ep_wait(exch, 0, world, epoch, DSV4_DEVERR_TIMEOUT_PEER, st)))
    return rc;
  if ((rc = launch_ep_unpack_p2p(exch, cap_tokens, T_own, k, H, e_begin, e_count, world,
                                 idx_local, w_local, ret_dst, st)))
    return rc;
  stage_mark(1, st);
  const SplitK sk = plan_split(p, ws);
  if ((rc = launch_route_plan(idx_local, T, k, e_count, 1, shared_rows, p.block_n, p.max_rows,
                              p.max_tiles, chunk_cnt, chunk_base, ctrl, counts, seg_start, tiles,
                              n_tiles, slot_token, slot_weight, st, sk.done1, split_counters(p))))
    return rc;
  stage_mark(2, st);
  if ((rc = launch_route_scatter(x_own, T_own, exch + kEpHeaderBytes, ep_row_bytes(H, k), idx_local,
                                 w_local, T, k, e_count, H, shared_rows, seg_start, chunk_base,
                                 ctrl, route_slot, slot_token, slot_weight, xq, xsf, nsm, st)))
    return rc;
  stage_mark(3, st);
  if ((rc = run_expert_gemms(L, tiles, n_tiles, slot_weight, xq, xsf, hq, hsf, O, H, p.max_rows,
                             p.max_tiles, p.block_n, L->expert_slot + e_begin, e_count, nsm, st, sk)))
    return rc;
  rc = launch_ep_return_p2p(O, H, k, route_slot, ret_dst, T * k, peer_bases, rank, world,
                            cap_tokens, epoch, nsm, st);
  stage_mark(6, st);
  return rc;
}

int dsv4_ep_combine_p2p(const dsv4_moe_layer* L, int rank, int world, const void* exchange,
                        const int* ret_pos, const int64_t* indices, int T_own, int cap_tokens,
                        int epoch, const void* workspace, long long workspace_bytes, void* y,
                        void* stream) {
  int rc = ep_check(L, rank, world);
  if (rc) return rc;
  if (T_own < 0 || T_own > cap_tokens || !exchange) return DSV4_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* exch = static_cast<const uint8_t*>(exchange);
  bind_device(exchange);
  // every owner's return rows are in place (waited for even with no tokens, so
  // the flags of this epoch are consumed in order)
  if ((rc = launch_ep_wait(exch, kEpRetFlagOff, world, epoch, DSV4_DEVERR_TIMEOUT_PEER, st)))
    return rc;
  if (T_own == 0) return DSV4_OK;
  if (!ret_pos || !indices || !y || !workspace) return DSV4_ERR_ARG;
  const int e_count = L->n_routed / world;
  const Plan p = make_plan(L, T_own + world * cap_tokens, e_count);
  if (workspace_bytes < p.total) return DSV4_ERR_WORKSPACE;
  const uint8_t* ws = static_cast<const uint8_t*>(workspace);
  const int* seg_start = reinterpret_cast<const int*>(ws + p.off[4]);
  const void* O = ws + p.off[14];
  return launch_combine(exch + ep_return_region_off(p.H, p.k, world, cap_tokens), p.H, ret_pos,
                        indices, T_own, p.k, p.S ? seg_start + e_count : nullptr, y, st, O);
}

int dsv4_ep_combine(const dsv4_moe_layer* L, int rank, int world, const void* ret_recv,
                    const int* ret_pos, const int64_t* indices, int T_own, int R,
                    const void* workspace, long long workspace_bytes, void* y, void* stream) {
  int rc = ep_check(L, rank, world);
  if (rc) return rc;
  if (T_own < 0 || R < 0) return DSV4_ERR_ARG;
  if (T_own == 0) return DSV4_OK;
  // every token has at least one route, so with T_own > 0 rows always return
  if (!ret_recv || !ret_pos || !indices || !y || !workspace) return DSV4_ERR_ARG;
  const int e_count = L->n_routed / world;
  const Plan p = make_plan(L, T_own + R, e_count);
  if (workspace_bytes < p.total) return DSV4_ERR_WORKSPACE;
  bind_device(y);
  const uint8_t* ws = static_cast<const uint8_t*>(workspace);
  const int* seg_start = reinterpret_cast<const int*>(ws + p.off[4]);
  const void* O = ws + p.off[14];
  // routed rows from the return buffer, the shared row from this rank's own output
  return launch_combine(ret_recv, p.H, ret_pos, indices, T_own, p.k,
                        p.S ? seg_start + e_count : nullptr, y, static_cast<cudaStream_t>(stream),
                        O);
}

}  // extern "C"
