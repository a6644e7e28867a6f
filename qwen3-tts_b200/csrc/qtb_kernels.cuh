// qtb_kernels.cuh -- the decode engine's device code.
//
// One persistent, cooperative kernel (decode_kernel) executes a "stage
// program": a flat list of stages separated by grid-wide barriers.  A talker
// step is 5 stages per layer (qwen_tts_talker.c:537-699):
//   GEMV qkv   (RMSNorm prologue, [q;k;v] rows fused into one matrix)
//   ATTN       (per-head QK RMSNorm + NeoX RoPE + bf16-truncating paged KV
//               append + split-K GQA attention + in-stage split combine)
//   GEMV o     (residual-add epilogue)
//   GEMV gu    (RMSNorm prologue, SwiGLU epilogue on the interleaved rows)
//   GEMV down  (residual-add epilogue)
// and a code-predictor frame is 16 such 5-layer passes with a greedy lm_head
// (GEMV with an argmax epilogue that also gathers the next pass's input
// embedding) between them (qwen_tts_code_predictor.c:926-1045).
//
// GEMV = weights x activations on the tensor cores (mma.sync m16n8k16).  At
// host upload every weight matrix is permuted into "fragment order": for each
// 16-row tile and each k-chunk, lane l's 16 bytes are exactly its A-fragment
// registers, so a warp streams 512 contiguous bytes per load and dequantizes
// in registers (bf16: none; int8: 1 PRMT + 1 HSUB2 per 2 weights; int4: 1 LOP3
// + 1 HSUB2 per 2 weights).  The f32 activation is split into hi + lo halves
// (bf16 or fp16, matching the weight operand type) which occupy two MMA
// columns, so the product keeps ~16-22 bits of activation precision with f32
// accumulation -- the reference's f32-activation semantics
// (qwen_tts_cuda_talker.cu:9-21) within a few 1e-6 relative.
#pragma once
#include "qtb_device.cuh"

namespace qtb {

constexpr int NTHREADS = 256;
constexpr int NWARPS = NTHREADS / 32;
constexpr int HD = 128;       // head_dim (Qwen3-TTS talker and CP)
constexpr int PAGE = 16;      // KV positions per page
constexpr int ATT_NBUF = 4;   // K/V page buffers in flight per CTA (small-batch programs)
constexpr int ATT_NBUF_MAX = 16;   // ... when the weight ring is idle (no small-batch GEMV stage)
constexpr int ATT_PAGE_BYTES = 2 * PAGE * HD * 2;   // one page of one KV head: K then V, bf16
constexpr long long WAIT_LIMIT_CYCLES = 500000000LL;  // ~0.25 s at 1.9 GHz

// Dynamic shared memory map (one CTA per SM):
//   [SM_W_OFF, +96 KB)   weight ring of the small-batch GEMV: NWSLOT slots
//                        filled by 1D bulk copies (TMA) by the weight streamer
//   [SM_X_OFF, +48 KB)   staged activation (small-batch GEMV) / K-V page
//                        ring + scratch of the attention stage
//   [SM_R_OFF, +12 KB)   1/rms, per-warp partial sums
// 156 KB in all, so with the static part the SM's unified L1/shared array can
// run the 164 KB shared-memory configuration and keep ~90 KB of L1 for the
// threads' stack frames (the stage functions are real calls).
// The large-batch GEMV path stages its activation slice from offset 0 (at
// most SMEM_X_BYTES); the weight streamer never runs past such a stage, so no
// bulk copy is in flight while it runs.
constexpr int WSLOT_BYTES = 16384;
constexpr int NWSLOT = 6;
constexpr int SM_W_OFF = 0;
constexpr int SM_X_OFF = NWSLOT * WSLOT_BYTES;
constexpr int SM_X2_BYTES = 48 * 1024;
constexpr int SM_R_OFF = SM_X_OFF + SM_X2_BYTES;
constexpr int SM_R_BYTES = 12 * 1024;
constexpr int SMEM_BYTES = SM_R_OFF + SM_R_BYTES;
// the last 1 KB of the R region receives a cluster partner's partial sums
constexpr int SM_PAIR_OFF = SM_R_OFF + SM_R_BYTES - 1024;
// Stage descriptors travel through a ring of NDESC shared-memory slots,
// bulk-copied NDESC - 1 stages ahead; the weight streamer looks at most
// STREAM_AHEAD stages past the last completed one (STREAM_AHEAD < NDESC keeps
// every descriptor it reads landed or pending in its slot's current phase).
constexpr int NDESC = 4;
constexpr int NCKPT = 32;     // profiling checkpoints per stage
constexpr int STREAM_AHEAD = NDESC - 1;
constexpr int SMEM_X_BYTES = 96 * 1024;

// tcgen05 GEMV stages (large batches, bf16 / int8 weights): the dynamic shared
// memory, from its first 1024-byte aligned byte, holds TC_NSLOT weight slots
// of one 128-row x 128-byte operand tile each, then TC_NSLOT activation slots
// of one N x 128-byte operand block each (before them, the prep phase's row
// buffer); a little scratch sits at TC_SCR_OFF.  These stages never share a
// program with the small-batch weight ring.
constexpr int TC_NSLOT = 3;
constexpr int TC_SLOT_BYTES = 16384;
constexpr int TC_XSLOT_BYTES = 32768;    // N <= 256 operand rows
constexpr int TC_XR_OFF = TC_NSLOT * TC_SLOT_BYTES;
constexpr int TC_SCR_OFF = 146 * 1024;   // past the slots + the 1 KB alignment slack
constexpr int TC_ACC_COLS = 256;         // one 128 x N (N <= 256) 32-bit accumulator
constexpr int TC_TMEM_COLS = 2 * TC_ACC_COLS;   // two: a tile is read back while the next accumulates
static_assert(TC_XR_OFF + TC_NSLOT * TC_XSLOT_BYTES + 1024 <= TC_SCR_OFF && TC_SCR_OFF + 4096 <= SMEM_BYTES,
              "tcgen05 stage smem map");

// Single-cluster schedule for small batches: the launch is one cluster of
// CL_G CTAs (cluster barriers instead of the grid barrier), and each warp
// streams its own GEMV weight pieces through two slots of CL_SLOT_BYTES in the
// weight-ring region, issuing the next stage's first pieces before the barrier.
constexpr int CL_G = 16;
constexpr int CL_SLOT_BYTES = NWSLOT * WSLOT_BYTES / (2 * NWARPS);
static_assert(CL_SLOT_BYTES % 1024 == 0, "per-warp weight slots");

enum StageKind { ST_GEMV = 1, ST_ATTN = 2, ST_EMBED = 3, ST_NORM = 4, ST_POS_INC = 5 };
enum Epi { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };
enum Fmt { FMT_BF16 = 0, FMT_INT8 = 1, FMT_Q4_0 = 2, FMT_INT4G = 3 };
enum ErrCode {
  ERR_NONE = 0, ERR_BARRIER_TIMEOUT = 1, ERR_MBAR_TIMEOUT = 2, ERR_BAD_PAGE = 3,
  ERR_BAD_POS = 4, ERR_BAD_CODE = 5, ERR_BAD_STAGE = 6
};

// Generation state of the codec head (the reference's frame loop, qwen_tts.c:
// 1648-1720), in device memory; read by the codec head's argmax epilogue and
// the position advance.  With enabled == 0 the head is a plain greedy argmax
// over its first eos_row rows.
struct GenState {
  int enabled;
  int eos_row;               // device row holding the EOS token's weights (rows past it are padding)
  int eos_token;             // 2150 (QWEN_TTS_CODEC_EOS)
  int vocab;                 // rep_count row length (the codebook)
  float rep_pen, rep_inv;    // repetition penalty and its reciprocal (as the reference's -ffast-math build uses)
  int *frame;                // [B] frames generated so far by the slot
  int *boost_start;          // [B] 2 x expected frames, or -1: no EOS boost
  int *done;                 // [B] 0 running, 1 sampled EOS in this frame, 2 stopped (parked)
  uint16_t *rep_count;       // [B][vocab] occurrences of each code0 so far
  // sampling (qwen_tts_sample): slots with temperature >= 1e-6 sample, the
  // others take the greedy maximum; `sampling` makes the codec head keep its
  // logits (after the rules above) for the sampler
  int sampling;
  int ld;                    // logits row stride (>= eos_row + 1)
  float *logits;             // [B][ld] codec-head logits of this frame
  float *temp;               // [B] temperature
  int *top_k;                // [B] top-k (<= 0: off)
  float *top_p;              // [B] top-p (>= 1: off)
  unsigned *rng;             // [B] state of the reference's LCG (qwen_set_seed / qwen_get_seed)
};

struct GemvArgs {
  const uint8_t *w;          // fragment-ordered weights
  const float *row_scale;    // int8: [rows]
  const uint8_t *gsz;        // int4: per (tile, 64-col chunk, group-of-4-lanes) scale(/zero)
  const float *bias;         // [rows] or null
  int fmt, rows, K, S;       // S = k-slices; units = rows/16 * S
  int nch;                   // MMA column chunks = ceil(P*B/8)
  int parts;                 // MMA columns per batch row: 2 (hi, lo) or 4 (hi, mid, lo, 0)
  int evict_last;            // keep these weights in L2 (code-predictor)
  int v2;                    // small-batch path: whole activation staged, weights TMA-streamed
  int tc;                    // large-batch path on tcgen05 (bf16 / int8 weights, see gemv_tc_t)
  int cl;                    // single-cluster schedule (gemv_cl_t): per-warp weight pieces
  const uint8_t *wtc;        // weights in 128-row x 128-byte swizzled tiles (tcgen05 operand layout)
  uint8_t *xop;              // tcgen05 path: the activation as the MMA's B operand (tc_prep_row)
  float *xsc;                // tcgen05 path: [64] part scale sx, [64] 1/rms of each batch row
  int sem_off;               // tcgen05 path: this stage's per-tile counters are sem[sem_off + tile]
  const float *x; int ldx;   // activation [B][ldx]
  const float *norm_w;       // RMSNorm gain [K] or null
  float eps;
  float *y; int ldy;
  int epi;
  float *ws; unsigned *sem;  // split-K partials [units][16][B] and per-tile counters
  // argmax epilogue
  unsigned long long *amax_ws; unsigned *amax_sem;
  int *codes; int code_stride;
  const uint16_t *emb_table; int emb_ld; int emb_rows; float *emb_out; int emb_out_ld;
  const GenState *gen;       // the codec head: its logit rules (codec_logit); null for the CP heads
};

struct AttnArgs {
  const float *qkv; int ld_qkv;
  float *out; int ld_out;
  const float *q_norm, *k_norm;
  const float *rope_cos, *rope_sin; int rope_len;
  const int *pos_ptr; int pos_const;
  const int *page_table; int pt_stride;
  uint16_t *kpool, *vpool; int n_pages;
  int n_heads, n_kv;
  float eps, scale;
  int max_splits, min_pps;
  float *ws; unsigned *sem;
  // nbuf: page buffers (ATT_NBUF, or ATT_NBUF_MAX in a program whose weight
  // ring is idle).  dyn: CTAs take work items from a grid-wide counter in the
  // dense order of attn_prefix instead of item = CTA + k * grid.
  int nbuf, dyn;
  // the host CPU's reciprocal-square-root seeds for the per-head QK RMSNorm
  // (qk_inv_rms), or null for IEEE 1 / sqrtf
  const unsigned *rsq_tab;
  // ATT_DECODE: append the token's K/V, then attend; ATT_APPEND: append only
  // (one item per slot and KV head); ATT_ATTEND: attend, causally by position,
  // to K/V appended before.  A prefill runs its prompt tokens as slots of one
  // sequence: all of them append first, then all attend.
  int mode;
  // prefill only: the prompt's K/V in f32 (pkv, layer `layer`).  APPEND
  // writes them there as well as into the pages; ATTEND reads positions from
  // the prompt's first one on from there, older ones from the pages.
  const struct PromptKV *pkv; int layer;
  // tensor-core decode attention (attn_pages_tc): tensor maps of this stack's
  // K and V pools ([layer][rows = page, kv head, position][128] bf16), pages
  // copied as 128-byte swizzled 16 x 64 boxes
  int tc; const void *kmap, *vmap;
};
enum AttnMode { ATT_DECODE = 0, ATT_APPEND = 1, ATT_ATTEND = 2 };

// The prompt of one prefill call in f32, [layer][n_kv][cap][HD] for K and V:
// positions p0 .. p0 + cap - 1.  The reference's prefill attends to its
// prompt's own K/V before the bf16 rounding of the cache
// (qwen_talker_prefill, qwen_tts_talker.c:904-914).
struct PromptKV { float *k, *v; int cap, p0; };

struct EmbedArgs {
  float *dst; int ld_dst; int dim;
  const float *fsrc; int fsrc_ld;
  int ntab;
  const uint16_t *tab[16]; int tab_ld[16]; int tab_rows[16];
  const int *code[16]; int code_stride[16];
  const float *add;
};

struct NormArgs { const float *x; int ldx; const float *w; float *y; int ldy; int dim; float eps; };
struct PosArgs { int *pos; const GenState *gen; };

// One stage of a program.  16-byte aligned and sized so the kernel can bulk-copy
// the next stage's descriptor into shared memory while the current one runs.
struct __align__(16) Stage {
  int kind;
  int B;
  union {
    GemvArgs g;
    AttnArgs a;
    EmbedArgs e;
    NormArgs n;
    PosArgs p;
  };
};
static_assert(sizeof(Stage) % 16 == 0, "stage descriptors are bulk-copied");

struct Ctl {
  unsigned bar_count;   // monotonic grid-barrier counter (zeroed before each launch)
  int err;              // first error code (same 8 bytes: one load polls both)
  int err_stage;        // stage index that raised it
  int err_info;
  unsigned att_work;    // attention work items taken (dynamic order; zeroed before each launch)
  unsigned ibar;        // tcgen05 stages: activation rows prepared (monotonic; zeroed before each launch)
  int trace_cta;        // the CTA whose intra-stage checkpoints a stage profile records
  int pad[57];
};

// Per-CTA kernel state, one copy in shared memory.  Fields are written by
// thread 0 only (at points separated from other threads' reads by a CTA
// barrier), except `local_err`, which any thread may set to 1.
struct V2Plan;

struct KCtx {
  unsigned epoch;
  unsigned page_ctr;    // K/V page buffers consumed so far (mbarrier phase source)
  unsigned wfill;       // weight-ring slot fills consumed so far (mbarrier phase source)
  unsigned att_issued;  // K/V page copies issued so far (one past the last)
  int att_nbuf;         // page buffers of the attention stages of this program
  unsigned att_base;    // ctl->att_work at the start of the current dynamic attention stage
  int att_first;        // first work item taken before the barrier, or -1
  int att_tot;          // its stage's item count (valid with att_first >= 0)
  int local_err;        // this thread has raised an error
  uint64_t pol_first, pol_last;
  uint64_t *bars;       // ATT_NBUF_MAX page-buffer mbarriers
  uint64_t *wbars;      // NWSLOT weight-slot mbarriers
  Ctl *ctl;
  int stage;
  long long *trace2;    // optional intra-stage checkpoints: [stage][NCKPT] clock64 of CTA trace_cta
  int trace_cta;
  unsigned long long *gtrace;  // optional [stage][cta] global time at arrival
  long long t_start;    // clock64 when this CTA left the last barrier
  // stage program and the weight streamer (streamer fields: thread 0 only)
  unsigned seq;         // running stage number: iteration * n_stages + stage
  unsigned n_total;     // stages in this launch
  int n_stages;
  Stage *dring;         // NDESC descriptor slots in shared memory
  V2Plan *pring;        // this CTA's plan entry for each descriptor slot
  uint64_t *dbars;      // their mbarriers
  unsigned w_issued;    // weight-ring fills issued so far
  unsigned w_free;      // fills whose slots have been read by every warp
  unsigned pf_seq;      // next stage the streamer looks at
  int pf_f;             // next fill of that stage
  int last;             // this CTA's arrival completed the current barrier
  uint64_t *pbar;       // receives the cluster partner's arrive (split stages)
  unsigned pair_ctr;    // split stages combined so far (pbar phase source)
  // tcgen05 GEMV stages (thread 0 issues copies and MMAs)
  uint32_t tmem;        // TMEM base address (TC_TMEM_COLS columns, allocated for the launch)
  uint64_t *tcfull;     // TC_NSLOT weight-slot mbarriers: bulk copy landed
  uint64_t *tcempty;    // ... the MMAs reading the slot completed (tcgen05.commit)
  uint64_t *tcacc;      // [2] the accumulator in TMEM buffer 0 / 1 is complete
  unsigned tc_issued;   // weight-slot fills issued so far in this launch
  unsigned tc_done;     // ... whose bulk copy has been waited for
  unsigned tc_committed;// tile accumulators committed so far (the g-th uses buffer g & 1)
  unsigned tc_waited;   // ... and waited for
  unsigned ibar_target; // ctl->ibar count that the current tcgen05 stage's prep completes
  // single-cluster schedule (a launch of one cluster of CL_G CTAs, see gemv_cl_t)
  int cl;               // this launch runs it: cluster barriers, per-warp weight pieces
  uint64_t *clbars;     // [2 * NWARPS] mbarriers of the warps' two weight slots
  unsigned cl_q[NWARPS];    // weight pieces each warp has consumed (lane 0 writes)
  unsigned cl_iss[NWARPS];  // ... and issued
  unsigned cl_pre[NWARPS];  // the stage whose first pieces were issued ahead (or ~0u)
  int cl_err;           // set (over distributed shared memory) by any CTA that raised an error
};

// Profiling checkpoint (CTA 0, thread 0) when stage tracing is on.
QTB_DEV void ckpt(const KCtx &kc, int i) {
  if (kc.trace2 && blockIdx.x == (unsigned)kc.trace_cta && threadIdx.x == 0) kc.trace2[(size_t)kc.stage * NCKPT + i] = clock64();
}
// Per-warp checkpoint (CTA 0, lane 0 of each warp): slot base + warp.
QTB_DEV void ckpt_w(const KCtx &kc, int base) {
  if (kc.trace2 && blockIdx.x == (unsigned)kc.trace_cta && (threadIdx.x & 31) == 0)
    kc.trace2[(size_t)kc.stage * NCKPT + base + (threadIdx.x >> 5)] = clock64();
}


QTB_DEV void raise_err(KCtx &kc, int code, int info) {
  kc.local_err = 1;
  if (atomicCAS(&kc.ctl->err, 0, code) == 0) {
    kc.ctl->err_stage = kc.stage;
    kc.ctl->err_info = info;
  }
}

// Grid-wide barrier on a monotonic counter, in two halves: grid_arrive here,
// grid_wait (which also runs the prefetch hook while it polls) next to the
// persistent kernel.  Bounded: the wait gives up (and raises
// ERR_BARRIER_TIMEOUT) after WAIT_LIMIT_CYCLES, or as soon as any CTA has
// raised an error, so a failing launch always returns.
QTB_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
QTB_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

QTB_DEV void grid_arrive(KCtx &kc) {
  __syncthreads();
  if (kc.cl) {
    // single-cluster launch: a CTA that raised an error tells every CTA of the
    // cluster (tag = this barrier's number + 1) before it arrives, so all of
    // them see it when this barrier completes and leave together
    if (kc.local_err && threadIdx.x < (unsigned)gridDim.x) {
      uint32_t r;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(&kc.cl_err)), "r"((uint32_t)threadIdx.x));
      asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(r), "r"((int)kc.epoch + 1) : "memory");
    }
    if (threadIdx.x == 0) kc.last = 0;
    __syncwarp();
    cluster_arrive();
    return;
  }
  // acq_rel: this CTA's writes (ordered before by bar.sync) happen-before every
  // CTA that acquires the final count; the CTA whose increment completes the
  // count acquires all the others' writes through the same RMW and needs no poll
  if (threadIdx.x == 0) {
    const unsigned target = (kc.epoch + 1u) * gridDim.x;
    kc.last = (atom_add_acq_rel_gpu(&kc.ctl->bar_count, 1u) + 1u == target) ? 1 : 0;
  }
}

// =========================================================== GEMV stage ====

// The f32 activation is carried as a sum of narrower parts, one MMA column
// each: fp16 hi + lo (22 mantissa bits) for the integer formats, bf16 hi +
// mid + lo (24 bits) or hi + lo (16 bits) for bf16 weights.  Returns part
// `part` of v0 and v1 packed as a pair.
template <bool F16>
QTB_DEV uint32_t split_pack(float v0, float v1, int part) {
  if (F16) {
    __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
    if (part == 1) {
      h0 = __float2half_rn(v0 - __half2float(h0));
      h1 = __float2half_rn(v1 - __half2float(h1));
    } else if (part > 1) {
      return 0u;
    }
    return (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
  } else {
    uint32_t r[2];
    const float v[2] = {v0, v1};
#pragma unroll
    for (int i = 0; i < 2; i++) {
      float rem = v[i];
      uint32_t b = f32_to_bf16_rn(rem);
      for (int k = 0; k < part && k < 3; k++) {
        rem -= __uint_as_float(b << 16);
        b = f32_to_bf16_rn(rem);
      }
      r[i] = (part > 2) ? 0u : b;
    }
    return r[0] | (r[1] << 16);
  }
}

// Per-batch 1/rms of the stage input (every CTA recomputes it; x is small).
QTB_DEV void stage_inv_rms(const GemvArgs &a, int B, float *s_inv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int b = warp; b < B; b += NWARPS) {
    const float *xb = a.x + (size_t)b * a.ldx;
    float ss = 0.f;
    // eight loads in flight per lane, summed in the same order as one at a time
    for (int i0 = lane * 4; i0 < a.K; i0 += 8 * 128) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = (i0 + 128 * u < a.K) ? ld_cg4(xb + i0 + 128 * u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; u++) ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
    }
    ss = warp_sum(ss);
    if (lane == 0) s_inv[b] = 1.0f / sqrtf(ss / (float)a.K + a.eps);
  }
}

QTB_DEV float norm_in(const GemvArgs &a, const float *s_inv, int b, int k, float v) {
  return a.norm_w ? (v * s_inv[b]) * __ldg(a.norm_w + k) : v;
}

// Stage the activation slice [k0, k0 + kslice) of every batch row into shared
// memory in B-fragment order (entry e = (kstep * nch + chunk) * ent + lane).
//
// Small-batch variant (B <= 4, B*K <= 8192): ONE pass over global memory.
// Thread i owns "quads" (batch b, k-step q, lane column tig): the 4 values
// x[b][16q + 2tig + {0, 1, 8, 9}], all loaded up front.  Sums of squares are
// reduced per batch row across the block, then every quad writes its P part
// entries (the lanes of its column group) and, for int4 weights, the per-32
// group sums (the 8 quads of a group sit in 8 consecutive lanes of one warp).
// Functions run once per stage on the critical path are real calls: one copy
// of their code stays in the SM's instruction cache across the stages.
#define QTB_CALL __device__ __noinline__
QTB_CALL void stream(KCtx &kc, char *smem, unsigned done, unsigned limit);

// MAXQ = quads (4 consecutive k of one batch row) per thread, B * K / 4 <=
// 256 * MAXQ; a separate function per MAXQ keeps the small cases' register
// footprint (and the caller's) small.
template <bool F16, int P, int MAXQ>
__device__ __noinline__ void stage_x_fused(const GemvArgs &a, int B, int ent, float *s_inv, float *s_xsum,
                                           uint2 *s_xf, bool want_xsum, KCtx &kc, char *smem) {
  const int K = a.K, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ks = K >> 4;
  const int nq = B * ks * 4;
  float v[MAXQ][4], nw[MAXQ][4];
  float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < MAXQ; i++) {
    const int t = tid + i * NTHREADS;
    if (t < nq) {
      const int tig = t & 3, q = (t >> 2) % ks, b = (t >> 2) / ks;
      const float *xb = a.x + (size_t)b * a.ldx + 16 * q + 2 * tig;
      const float2 p0 = __ldcg(reinterpret_cast<const float2 *>(xb));
      const float2 p1 = __ldcg(reinterpret_cast<const float2 *>(xb + 8));
      v[i][0] = p0.x; v[i][1] = p0.y; v[i][2] = p1.x; v[i][3] = p1.y;
      if (a.norm_w) {   // gains load alongside the activation (no dependency)
        const int k = 16 * q + 2 * tig;
        const float2 w0 = __ldg(reinterpret_cast<const float2 *>(a.norm_w + k));
        const float2 w1 = __ldg(reinterpret_cast<const float2 *>(a.norm_w + k + 8));
        nw[i][0] = w0.x; nw[i][1] = w0.y; nw[i][2] = w1.x; nw[i][3] = w1.y;
      }
    }
  }
  if (a.norm_w) {
    __shared__ float s_ss[NWARPS][4];
#pragma unroll
    for (int i = 0; i < MAXQ; i++) {
      const int t = tid + i * NTHREADS;
      if (t < nq) {
        const int b = (t >> 2) / ks;
        const float s2 = v[i][0] * v[i][0] + v[i][1] * v[i][1] + v[i][2] * v[i][2] + v[i][3] * v[i][3];
        // b is warp-uniform only when a warp's 32 quads share a row; add per row
#pragma unroll
        for (int bb = 0; bb < 4; bb++) ss[bb] += (b == bb) ? s2 : 0.f;
      }
    }
    ckpt(kc, 8);   // activation landed
    ckpt_w(kc, 16);
#pragma unroll
    for (int bb = 0; bb < 4; bb++) {
      const float w = warp_sum(ss[bb]);
      if (lane == 0) s_ss[warp][bb] = w;
    }
    __syncthreads();
    if (tid < 4) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < NWARPS; w++) tot += s_ss[w][tid];
      s_inv[tid] = rsqrtf(tot * __frcp_rn((float)K) + a.eps);   // within 2 ulp of 1 / sqrtf
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < MAXQ; i++) {
    const int t = tid + i * NTHREADS;
    float xs = 0.f;
    if (t < nq) {
      const int tig = t & 3, q = (t >> 2) % ks, b = (t >> 2) / ks;
      const int k = 16 * q + 2 * tig;
      (void)k;
      if (a.norm_w) {
        const float inv = s_inv[b];
        v[i][0] = (v[i][0] * inv) * nw[i][0];
        v[i][1] = (v[i][1] * inv) * nw[i][1];
        v[i][2] = (v[i][2] * inv) * nw[i][2];
        v[i][3] = (v[i][3] * inv) * nw[i][3];
      }
      xs = v[i][0] + v[i][1] + v[i][2] + v[i][3];
      // entries: column = b * P + part -> chunk j = col / 8, gid = col % 8
#pragma unroll
      for (int part = 0; part < P; part++) {
        const int col = b * P + part;
        const int j = col >> 3, gid = col & 7;
        const int e = (q * a.nch + j) * ent + gid * 4 + tig;
        s_xf[e] = make_uint2(split_pack<F16>(v[i][0], v[i][1], part), split_pack<F16>(v[i][2], v[i][3], part));
      }
    }
    if (want_xsum) {
      // 8 consecutive quads (k-steps 2g, 2g+1 x 4 columns) form group g
      xs += __shfl_xor_sync(0xffffffffu, xs, 1);
      xs += __shfl_xor_sync(0xffffffffu, xs, 2);
      xs += __shfl_xor_sync(0xffffffffu, xs, 4);
      if (t < nq && (t & 7) == 0) {
        const int q = (t >> 2) % ks, b = (t >> 2) / ks;
        s_xsum[b * (K >> 5) + (q >> 1)] = xs;
      }
    }
  }
}

template <bool F16>
// perm4: the int8 weight layout holds, per lane, 4 consecutive k of a 16-k
// step (the s8 MMA fragment); as an f16 MMA operand its logical k pairs
// (2tig, 2tig+1) and (8+2tig, 8+2tig+1) are physical k 4tig+{0,1} and
// 4tig+{2,3}, so the activation is staged in the same order.
QTB_DEV void stage_x(const GemvArgs &a, int B, int ent, int k0, int kslice, const float *s_inv,
                     float *s_xsum, uint2 *s_xf, bool want_xsum, bool perm4) {
  const int nch = a.nch, P = a.parts;
  const int ksteps = kslice >> 4;
  const int total = ksteps * nch * ent;
  if (ent == 32 && P == 2) {
    // large batches: coalesced float4 reads of each row's slice (eight in
    // flight per thread); a float4 holds two k pairs, each written as its two
    // parts into the fragment word that carries it (entry e = (q * nch + j) *
    // 32 + lane with column 8 j + gid = 2 b + part)
    const int nq4 = kslice >> 2, total4 = B * nq4;
    uint32_t *w = reinterpret_cast<uint32_t *>(s_xf);
    for (int base = threadIdx.x; base < total4; base += 8 * NTHREADS) {
      float4 v[8], nw[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int idx = base + u * NTHREADS;
        if (idx < total4) {
          const int b = idx / nq4, c = idx - b * nq4;
          v[u] = ld_cg4(a.x + (size_t)b * a.ldx + k0 + 4 * c);
          if (a.norm_w) nw[u] = __ldg(reinterpret_cast<const float4 *>(a.norm_w + k0 + 4 * c));
        }
      }
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int idx = base + u * NTHREADS;
        if (idx >= total4) break;
        const int b = idx / nq4, c = idx - b * nq4;
        float x4[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        if (a.norm_w) {
          const float r = s_inv[b];
          x4[0] = (x4[0] * r) * nw[u].x; x4[1] = (x4[1] * r) * nw[u].y;
          x4[2] = (x4[2] * r) * nw[u].z; x4[3] = (x4[3] * r) * nw[u].w;
        }
#pragma unroll
        for (int pr = 0; pr < 2; pr++) {
          const int kp = 2 * c + pr, q = kp >> 3, pi = kp & 7;
          const int tg = perm4 ? (pi >> 1) : (pi & 3), which = perm4 ? (pi & 1) : (pi >> 2);
#pragma unroll
          for (int lo = 0; lo < 2; lo++) {
            const int col = 2 * b + lo, jj = col >> 3, gg = col & 7;
            w[(((q * nch + jj) * 32) + gg * 4 + tg) * 2 + which] = split_pack<F16>(x4[2 * pr], x4[2 * pr + 1], lo);
          }
        }
      }
    }
    // MMA columns past the last batch row are zero
    const int pad = 8 * nch - 2 * B;
    for (int idx = threadIdx.x; idx < ksteps * pad * 4; idx += NTHREADS) {
      const int tg = idx & 3, r = idx >> 2, q = r / pad, col = 2 * B + (r - q * pad);
      s_xf[(q * nch + (col >> 3)) * 32 + (col & 7) * 4 + tg] = make_uint2(0u, 0u);
    }
  } else
  for (int e = threadIdx.x; e < total; e += NTHREADS) {
    const int l = e % ent;
    const int qj = e / ent;
    const int j = qj % nch, q = qj / nch;
    const int gid = l >> 2, tig = l & 3;
    const int col = 8 * j + gid;           // MMA column = batch * P + part
    const int b = col / P, lo = col % P;
    uint32_t r0 = 0, r1 = 0;
    if (b < B) {
      const int k = k0 + 16 * q + (perm4 ? 4 : 2) * tig, k2 = k + (perm4 ? 2 : 8);
      const float *xb = a.x + (size_t)b * a.ldx;
      float2 p0 = __ldcg(reinterpret_cast<const float2 *>(xb + k));
      float2 p1 = __ldcg(reinterpret_cast<const float2 *>(xb + k2));
      float v0 = norm_in(a, s_inv, b, k, p0.x), v1 = norm_in(a, s_inv, b, k + 1, p0.y);
      float v2 = norm_in(a, s_inv, b, k2, p1.x), v3 = norm_in(a, s_inv, b, k2 + 1, p1.y);
      r0 = split_pack<F16>(v0, v1, lo);
      r1 = split_pack<F16>(v2, v3, lo);
    }
    s_xf[e] = make_uint2(r0, r1);
  }
  if (want_xsum) {
    const int ng = kslice >> 5;
    for (int idx = threadIdx.x; idx < B * ng; idx += NTHREADS) {
      const int b = idx / ng, gl = idx - b * ng;
      const float *xb = a.x + (size_t)b * a.ldx;
      const int kb = k0 + gl * 32;
      float s = 0.f;
#pragma unroll 4
      for (int i = 0; i < 32; i += 2) {
        float2 p = __ldcg(reinterpret_cast<const float2 *>(xb + kb + i));
        s += norm_in(a, s_inv, b, kb + i, p.x);
        s += norm_in(a, s_inv, b, kb + i + 1, p.y);
      }
      s_xsum[idx] = s;
    }
  }
}

template <int FMT> struct FmtTraits;
template <> struct FmtTraits<FMT_BF16> { static constexpr int CK = 1; static constexpr int GSZ = 0; };
template <> struct FmtTraits<FMT_INT8> { static constexpr int CK = 2; static constexpr int GSZ = 0; };
template <> struct FmtTraits<FMT_Q4_0> { static constexpr int CK = 4; static constexpr int GSZ = 8; };
template <> struct FmtTraits<FMT_INT4G> { static constexpr int CK = 4; static constexpr int GSZ = 16; };

// Batch row held by a lane's accumulator pair in MMA column chunk j: with P
// columns per batch row, columns (2 tig, 2 tig + 1) belong to batch
// (8 j + 2 tig) / P.  With P = 4 two lanes (tig, tig ^ 1) share a batch row.
template <int P> QTB_DEV int col_batch(int j, int tig) { return P == 2 ? 4 * j + tig : 2 * j + (tig >> 1); }
template <int P> QTB_DEV bool col_owner(int tig) { return P == 2 || (tig & 1) == 0; }

// One 512-byte warp chunk of fragment-ordered weights (lane's 16 bytes in wv,
// its group scale/zero quad in gv for int4) times the staged activation.
// c = chunk index relative to the staged activation slice; bf16 / int8
// accumulate into acc, int4 applies its per-group scale and zero directly into
// res (groups are 32 columns = 2 k-steps).  xsum_n = groups in the slice.
template <int FMT, int NCH>
QTB_DEV void mma_chunk(const uint4 wv, const uint4 gv, int c, const uint2 *s_xf, int ent, const float *s_xsum,
                       int xsum_n, int B, float (&acc)[NCH][4], float (&res)[NCH][2], float (&acc2)[NCH][4]) {
  const int lane = threadIdx.x & 31, tig = lane & 3;
  const bool has_x = lane < ent;
  if (FMT == FMT_BF16) {
    const uint32_t A[4] = {wv.x, wv.y, wv.z, wv.w};
    const uint2 *xf = s_xf + (size_t)c * NCH * ent;
#pragma unroll
    for (int j = 0; j < NCH; j++) {
      uint2 bx = has_x ? xf[j * ent + lane] : make_uint2(0u, 0u);
      mma_bf16(acc[j], A, bx.x, bx.y);
    }
  } else if (FMT == FMT_INT8) {
    // s8 MMA layout (words: row gid k0..3, row gid+8 k0..3, then k16..19),
    // read as two f16 MMAs over the perm4 k order
    const uint32_t wd[4] = {wv.x ^ 0x80808080u, wv.y ^ 0x80808080u, wv.z ^ 0x80808080u, wv.w ^ 0x80808080u};
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const uint32_t A[4] = {i8x2_to_f16x2(wd[2 * q], 0x4140), i8x2_to_f16x2(wd[2 * q + 1], 0x4140),
                             i8x2_to_f16x2(wd[2 * q], 0x4342), i8x2_to_f16x2(wd[2 * q + 1], 0x4342)};
      const uint2 *xf = s_xf + (size_t)(2 * c + q) * NCH * ent;
#pragma unroll
      for (int j = 0; j < NCH; j++) {
        uint2 bx = has_x ? xf[j * ent + lane] : make_uint2(0u, 0u);
        if (q == 0) mma_f16(acc[j], A, bx.x, bx.y);   // two independent chains
        else mma_f16(acc2[j], A, bx.x, bx.y);
      }
    }
  } else {
    // int4: two groups of 32 columns per chunk.
    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int gh = 0; gh < 2; gh++) {
      float sc0, sc1, z0, z1;
      sc0 = half_bits_to_f32(gh ? (gv.x >> 16) : (gv.x & 0xffffu));
      sc1 = half_bits_to_f32(gh ? (gv.y >> 16) : (gv.y & 0xffffu));
      if (FMT == FMT_Q4_0) {
        z0 = 8.f; z1 = 8.f;
      } else {
        z0 = half_bits_to_f32(gh ? (gv.z >> 16) : (gv.z & 0xffffu));
        z1 = half_bits_to_f32(gh ? (gv.w >> 16) : (gv.w & 0xffffu));
      }
      const int gl = 2 * c + gh;   // group index within the slice
#pragma unroll
      for (int j = 0; j < NCH; j++) {
        float cg[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int qq = 0; qq < 2; qq++) {
          const uint32_t w = wd[2 * gh + qq];
          const uint32_t A[4] = {u4x2_to_f16x2(w), u4x2_to_f16x2(w >> 4), u4x2_to_f16x2(w >> 8),
                                 u4x2_to_f16x2(w >> 12)};
          const uint2 *xf = s_xf + (size_t)(4 * c + 2 * gh + qq) * NCH * ent;
          uint2 bx = has_x ? xf[j * ent + lane] : make_uint2(0u, 0u);
          mma_f16(cg, A, bx.x, bx.y);
        }
        const int b = 4 * j + tig;
        const float xs = (b < B) ? s_xsum[b * xsum_n + gl] : 0.f;
        res[j][0] += sc0 * ((cg[0] + cg[1]) - z0 * xs);
        res[j][1] += sc1 * ((cg[2] + cg[3]) - z1 * xs);
      }
    }
  }
}

// Fold the MMA accumulators into per-row results (hi + lo (+ mid) columns).
template <int FMT, int NCH, int P>
QTB_DEV void acc_finish(float (&acc)[NCH][4], float (&res)[NCH][2]) {
  if (FMT == FMT_BF16 || FMT == FMT_INT8) {
#pragma unroll
    for (int j = 0; j < NCH; j++) {
      res[j][0] = acc[j][0] + acc[j][1];
      res[j][1] = acc[j][2] + acc[j][3];
      if (P == 4) {
        res[j][0] += __shfl_xor_sync(0xffffffffu, res[j][0], 1);
        res[j][1] += __shfl_xor_sync(0xffffffffu, res[j][1], 1);
      }
    }
  }
}

// One warp computes one unit: 16 rows x kslice columns, all batch columns.
// res[j][0] / res[j][1] = rows (16t + gid) / (16t + gid + 8) for batch
// col_batch<P>(j, tig).
template <int FMT, int NCH, int P>
QTB_DEV void gemv_unit(const GemvArgs &a, int B, int t, int s, int kslice, const uint2 *s_xf,
                       int ent, const float *s_xsum, float (&res)[NCH][2], const KCtx &kc) {
  using Tr = FmtTraits<FMT>;
  constexpr int CK = Tr::CK;
  // loads in flight per lane: the warp's chunk stream is latency-bound, so as
  // deep as the registers allow -- less deep
  // for large ones (the accumulators need the registers; int8 keeps two sets)
  constexpr int PD = NCH >= 8 ? (FMT == FMT_BF16 ? 8 : 2) : (NCH >= 4 ? 4 : 8);
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int nck_total = a.K / (16 * CK);
  const int nck = kslice / (16 * CK);
  const size_t cbase = (size_t)t * nck_total + (size_t)s * nck;
  const uint8_t *wp = a.w + cbase * 512 + lane * 16;
  const uint8_t *gp = Tr::GSZ ? a.gsz + cbase * (8 * Tr::GSZ) + gid * Tr::GSZ : nullptr;
  const uint64_t pol = a.evict_last ? kc.pol_last : kc.pol_first;
  const bool has_x = lane < ent;

  float acc[NCH][4], acc2[NCH][4];
#pragma unroll
  for (int j = 0; j < NCH; j++) {
    acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    acc2[j][0] = acc2[j][1] = acc2[j][2] = acc2[j][3] = 0.f;
    res[j][0] = res[j][1] = 0.f;
  }

  uint4 wbuf[PD];
  uint4 gbuf[PD];
#pragma unroll
  for (int i = 0; i < PD; i++) {
    if (i < nck) {
      wbuf[i] = ld_stream_hint(wp + (size_t)i * 512, pol);
      if (Tr::GSZ == 8) { uint2 g = ld_nc_u2(gp + (size_t)i * 64); gbuf[i] = make_uint4(g.x, g.y, 0, 0); }
      if (Tr::GSZ == 16) gbuf[i] = ld_nc_u4(gp + (size_t)i * 128);
    }
  }
  for (int c0 = 0; c0 < nck; c0 += PD) {
#pragma unroll
    for (int i = 0; i < PD; i++) {
      const int c = c0 + i;
      if (c < nck) {
        const uint4 wv = wbuf[i];
        const uint4 gv = gbuf[i];
        if (c + PD < nck) {
          wbuf[i] = ld_stream_hint(wp + (size_t)(c + PD) * 512, pol);
          if (Tr::GSZ == 8) { uint2 g = ld_nc_u2(gp + (size_t)(c + PD) * 64); gbuf[i] = make_uint4(g.x, g.y, 0, 0); }
          if (Tr::GSZ == 16) gbuf[i] = ld_nc_u4(gp + (size_t)(c + PD) * 128);
        }
        mma_chunk<FMT, NCH>(wv, gv, c, s_xf, ent, s_xsum, kslice >> 5, B, acc, res, acc2);
      }
    }
  }
  if (FMT == FMT_INT8) {   // (only int8 uses the second set)
#pragma unroll
    for (int j = 0; j < NCH; j++)
#pragma unroll
      for (int e2 = 0; e2 < 4; e2++) acc[j][e2] += acc2[j][e2];
  }
  acc_finish<FMT, NCH, P>(acc, res);
}

QTB_DEV unsigned long long amax_key(float v, int row) {
  return ((unsigned long long)float_order_key(v) << 32) | (unsigned long long)(0xffffffffu - (unsigned)row);
}
// The codec head's logit of device row `row` for slot b, as the reference's
// frame loop forms it before greedy sampling (qwen_tts.c:1650-1676 and the
// repetition penalty of qwen_tts_sample, qwen_tts_sampling.c:160-181): clipped
// to +-100; special tokens masked (-1e30) except EOS, which is masked for the
// slot's first two frames and boosted by min(0.5 (frame - boost_start), 10)
// after its boost start; then every earlier occurrence of the token scales it
// by 1 / penalty (positive) or penalty (otherwise), one rounding each.
QTB_DEV float codec_rules(const GenState *gs, int b, int row, float v) {
  if (v > 100.0f) v = 100.0f;
  if (v < -100.0f) v = -100.0f;
  const int frame = __ldcg(gs->frame + b);
  if (row == gs->eos_row) {
    if (frame < 2) return -1e30f;
    const int bs = __ldcg(gs->boost_start + b);
    if (bs >= 0 && frame > bs) {
      float boost = 0.5f * (float)(frame - bs);
      if (boost > 10.0f) boost = 10.0f;
      v += boost;
    }
    return v;
  }
  const int c = __ldcg(gs->rep_count + (size_t)b * gs->vocab + row);
  for (int i = 0; i < c; i++) v = (v > 0.0f) ? __fmul_rn(v, gs->rep_inv) : __fmul_rn(v, gs->rep_pen);
  return v;
}
QTB_DEV float codec_logit(const GenState *gs, int b, int row, float v) {
  if (row > gs->eos_row) return -1e30f;
  if (!gs->enabled) return row == gs->eos_row ? -1e30f : v;
  v = codec_rules(gs, b, row, v);
  if (gs->sampling) __stcg(gs->logits + (size_t)b * gs->ld + row, v);
  return v;
}

// Temperature / top-k / top-p sampling of slot b's codec-head logits (rows
// 0 .. eos_row, the rules above applied), as the reference's qwen_tts_sample
// does it after its repetition penalty (qwen_tts_sampling.c:52-202): softmax
// at the temperature (x * (1 / T), exp, x * (1 / sum)), top-k keeping every
// value >= the k-th largest, top-p keeping the largest values up to the first
// whose running sum passes p, renormalisation, then one draw of the
// reference's LCG (state * 1103515245 + 12345, 15 bits / 32768) against the
// running sum in row order.  One warp; row i sits in lane i % 32, register
// i / 32.  The sums run in a different order than the reference's loops (to
// the last bits of f32); the k-th largest and the top-p cut are found by a
// bitwise search over the non-negative probabilities' bit patterns.  Returns
// the row drawn (eos_row = EOS).
constexpr int SAMPLE_MAX_ROWS = 2176;
QTB_DEV int sample_codec(const GenState *gs, int b) {
  constexpr int PER = SAMPLE_MAX_ROWS / 32;
  const int lane = threadIdx.x & 31;
  const int n = gs->eos_row + 1;
  const float *lg = gs->logits + (size_t)b * gs->ld;
  const float temp = __ldcg(gs->temp + b);
  const int top_k = __ldcg(gs->top_k + b);
  const float top_p = __ldcg(gs->top_p + b);
  float p[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const int r = i * 32 + lane;
    p[i] = r < n ? __ldcg(lg + r) : -INFINITY;
    mx = fmaxf(mx, p[i]);
  }
  mx = warp_max(mx);
  const float inv_t = 1.0f / temp;
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const int r = i * 32 + lane;
    p[i] = r < n ? expf((p[i] - mx) * inv_t) : 0.f;
    sum += p[i];
  }
  sum = warp_sum(sum);
  float inv = 1.0f / sum;
#pragma unroll
  for (int i = 0; i < PER; i++) p[i] *= inv;
  // the largest bit pattern t whose count / mass of {p >= t} still meets the bar
  auto search = [&](bool by_mass, float bar) -> unsigned {
    unsigned thr = 0u;
    for (int bit = 30; bit >= 0; bit--) {
      const unsigned cand = thr | (1u << bit);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < PER; i++)
        if (__float_as_uint(p[i]) >= cand) acc += by_mass ? p[i] : 1.0f;
      acc = warp_sum(acc);
      if (by_mass ? (acc > bar) : (acc >= bar)) thr = cand;
    }
    return thr;
  };
  if (top_k > 0 && top_k < n) {
    const unsigned thr = search(false, (float)top_k);
#pragma unroll
    for (int i = 0; i < PER; i++)
      if (__float_as_uint(p[i]) < thr) p[i] = 0.f;
  }
  if (top_p < 1.0f && top_p > 0.0f) {
    const unsigned thr = search(true, top_p);
#pragma unroll
    for (int i = 0; i < PER; i++)
      if (__float_as_uint(p[i]) < thr) p[i] = 0.f;
  }
  sum = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) sum += p[i];
  sum = warp_sum(sum);
  if (sum > 0.f) {
    inv = 1.0f / sum;
#pragma unroll
    for (int i = 0; i < PER; i++) p[i] *= inv;
  }
  unsigned st = __ldcg(gs->rng + b);
  st = st * 1103515245u + 12345u;
  const float u = (float)((st >> 16) & 0x7FFFu) / 32768.0f;
  // the first row whose running sum passes u; past the end, the last row
  // with a non-zero probability (the reference then returns its last row)
  float run = 0.f;
  int pick = -1, last_nz = -1;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    float c = p[i];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, c, o);
      if (lane >= o) c += t;
    }
    const float tot = run + c;
    const unsigned hit = __ballot_sync(0xffffffffu, pick < 0 && u < tot);
    if (pick < 0 && hit) pick = i * 32 + (__ffs(hit) - 1);
    const unsigned nz = __ballot_sync(0xffffffffu, p[i] > 0.f);
    if (nz) last_nz = i * 32 + (31 - __clz(nz));
    run += __shfl_sync(0xffffffffu, c, 31);
  }
  if (lane == 0) gs->rng[b] = st;
  __syncwarp();
  return pick >= 0 ? pick : last_nz;
}

QTB_DEV unsigned long long shfl_xor_u64(unsigned long long v, int m) {
  unsigned lo = (unsigned)v, hi = (unsigned)(v >> 32);
  lo = __shfl_xor_sync(0xffffffffu, lo, m);
  hi = __shfl_xor_sync(0xffffffffu, hi, m);
  return ((unsigned long long)hi << 32) | lo;
}

// Epilogue for the 16 final rows of tile t (called by exactly one warp).
template <int NCH, int P>
QTB_DEV void gemv_epilogue(const GemvArgs &a, int B, int t, int T, float (&res)[NCH][2], KCtx &kc) {
  const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int j = 0; j < NCH; j++) {
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int row = 16 * t + gid + 8 * r;
      float v = res[j][r];
      if (a.row_scale) v = __ldg(a.row_scale + row) * v;
      if (a.bias) v += __ldg(a.bias + row);
      res[j][r] = v;
    }
  }
  if (a.epi == EPI_ARGMAX) {
#pragma unroll
    for (int j = 0; j < NCH; j++) {
      const int bj = col_batch<P>(j, tig);
      const float v0 = (a.gen && bj < B) ? codec_logit(a.gen, bj, 16 * t + gid, res[j][0]) : res[j][0];
      const float v1 = (a.gen && bj < B) ? codec_logit(a.gen, bj, 16 * t + gid + 8, res[j][1]) : res[j][1];
      unsigned long long k0 = amax_key(v0, 16 * t + gid), k1 = amax_key(v1, 16 * t + gid + 8);
      unsigned long long k = k0 > k1 ? k0 : k1;
#pragma unroll
      for (int m = 4; m < 32; m <<= 1) {
        unsigned long long o = shfl_xor_u64(k, m);
        k = o > k ? o : k;
      }
      const int b = col_batch<P>(j, tig);
      if (gid == 0 && b < B && col_owner<P>(tig)) a.amax_ws[(size_t)t * B + b] = k;
    }
    __syncwarp();
    unsigned old = 0;
    if (lane == 0) { __threadfence(); old = atomicAdd(a.amax_sem, 1u); }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != (unsigned)(T - 1)) return;
    __threadfence();
    for (int b0 = 0; b0 < B; b0 += 32) {
      const int b = b0 + lane;
      int code = 0;
      if (b < B) {
        unsigned long long best = 0ull;
        for (int tt = 0; tt < T; tt++) {
          unsigned long long k = __ldcg(a.amax_ws + (size_t)tt * B + b);
          best = k > best ? k : best;
        }
        code = (int)(0xffffffffu - (unsigned)(best & 0xffffffffull));
        a.codes[(size_t)b * a.code_stride] = code;
      }
      if (a.emb_table) {
        const int nb = min(32, B - b0);
        for (int bb = 0; bb < nb; bb++) {
          int cb = __shfl_sync(0xffffffffu, code, bb);
          if (cb < 0 || cb >= a.emb_rows) { if (lane == 0) raise_err(kc, ERR_BAD_CODE, cb); cb = 0; }
          const uint16_t *row = a.emb_table + (size_t)cb * a.emb_ld;
          float *dst = a.emb_out + (size_t)(b0 + bb) * a.emb_out_ld;
          for (int i = lane * 8; i < a.emb_ld; i += 256) {
            uint4 v = ld_nc_u4(row + i);
            float4 lo4 = make_float4(bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y));
            float4 hi4 = make_float4(bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w));
            __stcg(reinterpret_cast<float4 *>(dst + i), lo4);
            __stcg(reinterpret_cast<float4 *>(dst + i + 4), hi4);
          }
        }
      }
    }
    if (lane == 0) *a.amax_sem = 0u;
    return;
  }
  const bool owner = col_owner<P>(tig);
#pragma unroll
  for (int j = 0; j < NCH; j++) {
    const int b = col_batch<P>(j, tig);
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int row = 16 * t + gid + 8 * r;
      const float v = res[j][r];
      if (a.epi == EPI_SWIGLU) {
        const float up = __shfl_xor_sync(0xffffffffu, v, 4);
        if ((gid & 1) == 0 && b < B && owner) {
          const float g = v;
          __stcg(a.y + (size_t)b * a.ldy + (row >> 1), g / (1.0f + expf(-g)) * up);
        }
      } else if (b < B && owner) {
        float *yp = a.y + (size_t)b * a.ldy + row;
        if (a.epi == EPI_RESID) __stcg(yp, __ldcg(yp) + v);
        else __stcg(yp, v);
      }
    }
  }
}

template <int FMT, int NCH, int P>
__device__ __noinline__ void gemv_stage_t(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  const int T = a.rows >> 4;
  const int S = a.S;
  const int U = T * S;
  const int kslice = a.K / S;
  const int W = gridDim.x * NWARPS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int ent = 4 * min(8, P * B);
  constexpr bool F16 = (FMT != FMT_BF16);
  constexpr bool XSUM = (FMT == FMT_Q4_0 || FMT == FMT_INT4G);

  float *s_inv = reinterpret_cast<float *>(smem);                 // 64 floats
  float *s_xsum = s_inv + 64;                                     // B * kslice/32 (int4)
  const int xsum_n = XSUM ? ((B * (kslice >> 5) + 3) & ~3) : 0;
  uint2 *s_xf = reinterpret_cast<uint2 *>(s_xsum + xsum_n);

  bool inv_done = false;
  for (int base = blockIdx.x * NWARPS; base < U; base += W) {
    if (a.norm_w && !inv_done) { stage_inv_rms(a, B, s_inv); __syncthreads(); inv_done = true; }
    ckpt(kc, 12);
    const int s = base / T;
    stage_x<F16>(a, B, ent, s * kslice, kslice, s_inv, s_xsum, s_xf, XSUM, FMT == FMT_INT8);
    __syncthreads();
    ckpt(kc, 13);
    const int u = base + warp;
    if (u < U) {
      const int t = u - s * T;
      float res[NCH][2];
      gemv_unit<FMT, NCH, P>(a, B, t, s, kslice, s_xf, ent, s_xsum, res, kc);
      ckpt(kc, 14);
      bool finish = true;
      if (S > 1) {
#pragma unroll
        for (int j = 0; j < NCH; j++) {
          const int b = col_batch<P>(j, tig);
          if (b < B && col_owner<P>(tig)) {
            __stcg(a.ws + ((size_t)u * 16 + gid) * B + b, res[j][0]);
            __stcg(a.ws + ((size_t)u * 16 + gid + 8) * B + b, res[j][1]);
          }
        }
        __syncwarp();
        unsigned old = 0;
        if (lane == 0) { __threadfence(); old = atomicAdd(a.sem + t, 1u); }
        old = __shfl_sync(0xffffffffu, old, 0);
        finish = (old == (unsigned)(S - 1));
        ckpt(kc, 15);
        if (finish) {
          __threadfence();
          // the S partials in slice order; two slices' loads in flight at a
          // time (S is a power of two)
#pragma unroll
          for (int j = 0; j < NCH; j++) res[j][0] = res[j][1] = 0.f;
          for (int ss = 0; ss < S; ss += 2) {
            float l[2][NCH][2];
#pragma unroll
            for (int q = 0; q < 2; q++) {
              const size_t uu = (size_t)(ss + q) * T + t;
#pragma unroll
              for (int j = 0; j < NCH; j++) {
                const int b = col_batch<P>(j, tig);
                const bool ok = b < B && ss + q < S;
                l[q][j][0] = ok ? __ldcg(a.ws + (uu * 16 + gid) * B + b) : 0.f;
                l[q][j][1] = ok ? __ldcg(a.ws + (uu * 16 + gid + 8) * B + b) : 0.f;
              }
            }
#pragma unroll
            for (int q = 0; q < 2; q++)
#pragma unroll
              for (int j = 0; j < NCH; j++) {
                res[j][0] += l[q][j][0];
                res[j][1] += l[q][j][1];
              }
          }
          if (lane == 0) a.sem[t] = 0u;
        }
      }
      ckpt(kc, 16);
      if (finish) gemv_epilogue<NCH, P>(a, B, t, T, res, kc);
      ckpt(kc, 17);
    }
    __syncthreads();
  }
}

// ============================================ GEMV stage, small batches ====
//
// Used when the whole activation (B rows x K) fits the staging region.  Each
// CTA owns a run of whole 16-row tiles, so its weights are ONE contiguous byte
// range of the fragment-ordered matrix.  Thread 0 is also the CTA's weight
// streamer: it bulk-copies those ranges, stage after stage in program order,
// into the NWSLOT-slot ring as slots free up -- typically while the grid
// barriers of the stages before are still pending -- so a stage usually finds
// its weights already in shared memory.  Warps split the CTA's chunk stream
// evenly, keep one partial per (tile, warp) in shared memory, and the CTA sums
// them in warp order (deterministic).

struct V2Sched {
  int t0, nt;   // first tile and tile count of this CTA
  int kb, kc;   // first chunk and chunk count within each tile
  int L;        // chunks = nt * kc
  int cps;      // chunks per ring slot
  int nfill;    // slot fills = ceil(L / cps)
};

// A CTA's share of a small-batch GEMV stage, computed on the host for every
// (stage, CTA) and bulk-copied with the stage descriptor, so the kernel does
// no integer division to find it: whole 16-row tiles t0 .. t0+nt-1 (when
// there are fewer tiles than CTAs the rest idle -- the weights are streamed
// ahead, so a CTA holding two tiles' worth costs less than a cross-CTA
// reduction would), L chunks of 512 bytes in nfill ring fills.
// pair: 0, or for an int8 stage without a norm and with fewer than half as
// many tiles as CTAs, the tile's K is cut in two between the CTAs of one
// 2-CTA cluster (CTAs 2u, 2u+1 for tile u): 1 = the first half, which also
// adds the second half's sums (sent over distributed shared memory, in piece
// order: deterministic) and runs the epilogue, 2 = the second half.
struct __align__(16) V2Plan {
  int t0, nt, L, nfill;
  int kb, kc, pair, pad;
};
static_assert(sizeof(V2Plan) == 32, "plans are bulk-copied");

template <int FMT>
QTB_HOST_DEV constexpr int v2_cps() { return WSLOT_BYTES / (512 + 8 * FmtTraits<FMT>::GSZ); }

// `pairs`: the launch runs in 2-CTA clusters, so K may be split across a pair.
QTB_HOST_DEV V2Plan v2_plan(int fmt, int rows, int K, bool has_norm, int epi, int cta, int G, bool pairs) {
  const int gsz = fmt == FMT_Q4_0 ? 8 : (fmt == FMT_INT4G ? 16 : 0);
  const int ck = fmt == FMT_BF16 ? 1 : (fmt == FMT_INT8 ? 2 : 4);
  const int T = rows >> 4, nck = K / (16 * ck), cps = WSLOT_BYTES / (512 + 8 * gsz);
  V2Plan p;
  p.pad = 0;
  if (pairs && fmt == FMT_INT8 && !has_norm && epi != EPI_ARGMAX && 2 * T <= G && nck >= 8) {
    const int u = cta >> 1, h = cta & 1, n4 = nck >> 2;
    p.t0 = u < T ? u : 0;
    p.nt = u < T ? 1 : 0;
    p.kb = h ? 4 * (n4 / 2) : 0;
    p.kc = h ? nck - 4 * (n4 / 2) : 4 * (n4 / 2);
    p.pair = p.nt ? 1 + h : 0;
    p.L = p.nt * p.kc;
  } else {
    p.t0 = (int)((long long)cta * T / G);
    p.nt = (int)((long long)(cta + 1) * T / G) - p.t0;
    p.kb = 0;
    p.kc = nck;
    p.pair = 0;
    p.L = p.nt * nck;
  }
  p.nfill = (p.L + cps - 1) / cps;
  return p;
}

template <int FMT>
QTB_DEV V2Sched v2_sched(const GemvArgs &a, const V2Plan &p) {
  using Tr = FmtTraits<FMT>;
  V2Sched s;
  s.cps = v2_cps<FMT>();
  s.t0 = p.t0;
  s.nt = p.nt;
  s.kb = p.kb;
  s.kc = p.kc;
  (void)Tr::CK;
  s.L = p.L;
  s.nfill = p.nfill;
  return s;
}

// One warp: bulk-copy slot fills [f0, f1) (at most NWSLOT) of this CTA's range
// into the ring, lane i issuing fill f0 + i (the copies are issued in
// parallel: one bulk copy costs a thread ~250 cycles to issue); fill f0 is the
// launch's fill number ctr0 (slot ctr0 % NWSLOT).
template <int FMT>
QTB_DEV void v2_issue(const GemvArgs &a, const V2Sched &s, int f0, int f1, unsigned ctr0, const KCtx &kc,
                      char *smem) {
  using Tr = FmtTraits<FMT>;
  const int nck = a.K / (16 * Tr::CK);
  const size_t cbase = (size_t)s.t0 * nck + s.kb;
  const uint64_t pol = a.evict_last ? kc.pol_last : kc.pol_first;
  const int f = f0 + (int)(threadIdx.x & 31);
  if (f < f1) {
    fence_proxy_async_smem();   // the slot was last read through the generic proxy
    const unsigned ctr = ctr0 + (unsigned)(f - f0);
    const int slot = (int)(ctr % NWSLOT);
    const int c0 = f * s.cps, n = min(s.cps, s.L - c0);
    char *dst = smem + SM_W_OFF + slot * WSLOT_BYTES;
    uint64_t *bar = kc.wbars + slot;
    const uint32_t wbytes = (uint32_t)n * 512u, gbytes = (uint32_t)n * 8u * Tr::GSZ;
    mbar_arrive_expect_tx(bar, wbytes + gbytes);
    bulk_g2s_hint(dst, a.w + (cbase + c0) * 512, wbytes, bar, pol);
    if (Tr::GSZ) bulk_g2s_hint(dst + s.cps * 512, a.gsz + (cbase + c0) * (8 * Tr::GSZ), gbytes, bar, pol);
  }
}

// Streamer step for one small-batch GEMV stage (one warp): issue as many of
// this CTA's remaining fills as the ring has free slots.  True once all are
// issued.
template <int FMT>
QTB_DEV bool stream_gemv(const GemvArgs &a, const V2Plan &p, KCtx &kc, char *smem) {
  const V2Sched s = v2_sched<FMT>(a, p);
  if (s.nfill == 0) return true;
  const int pf_f = kc.pf_f;
  const int room = NWSLOT - (int)(kc.w_issued - kc.w_free);
  const int n = min(s.nfill - pf_f, room);
  if (n > 0) v2_issue<FMT>(a, s, pf_f, pf_f + n, kc.w_issued, kc, smem);
  __syncwarp();
  if ((threadIdx.x & 31) == 0 && n > 0) {
    kc.pf_f = pf_f + n;
    kc.w_issued += (unsigned)n;
  }
  __syncwarp();
  return pf_f + max(n, 0) >= s.nfill;
}

// Ask L2 for a coming GEMV stage's small operands (RMSNorm gains, this CTA's
// row scales and bias), so its activation staging and epilogue hit L2.
QTB_DEV void prefetch_gemv_operands(const GemvArgs &a, const V2Plan &p) {
  if (p.nt == 0) return;
  if (a.norm_w) prefetch_l2(a.norm_w, (uint32_t)a.K * 4u);
  if (a.row_scale) prefetch_l2(a.row_scale + 16 * p.t0, (uint32_t)p.nt * 64u);
  if (a.bias) prefetch_l2(a.bias + 16 * p.t0, (uint32_t)p.nt * 64u);
}

// The weight streamer, run by all 32 lanes of one warp.  Walks the stage
// program ahead of the stage being computed and bulk-copies the weights of
// coming small-batch GEMV stages into the ring as slots free up.  Fills are
// issued and consumed in program order, so the launch's n-th fill always lands
// in slot n % NWSLOT.  `done` = stages this CTA has completed; stages before
// `limit` are looked at.  The streamer stops at a descriptor that has not
// landed, at a large-batch GEMV stage that has not run yet (that path uses the
// ring region for its activation), and STREAM_AHEAD stages past `done`.
// Callers look one stage ahead only once the current stage's activation loads
// are in flight, so the bulk traffic queues behind them.  Only lane 0 writes
// the streamer state; __syncwarp orders it for the other lanes.
QTB_CALL void stream(KCtx &kc, char *smem, unsigned done, unsigned limit) {
  const int lane = threadIdx.x & 31;
  if (kc.cl) return;   // the single-cluster GEMV stages stream their own weights
  // A completed stage has no fills left to issue (each GEMV stage issues its
  // own before reading them), and its descriptor slot may already hold a later
  // stage: never look behind `done`.
  if (kc.pf_seq < done) {
    __syncwarp();
    if (lane == 0) {
      kc.pf_seq = done;
      kc.pf_f = 0;
    }
    __syncwarp();
  }
  while (true) {
    const unsigned k = kc.pf_seq;
    if (!(k < kc.n_total && k < limit && k < done + STREAM_AHEAD)) break;
    const int slot = (int)(k % NDESC);
    if (!mbar_test(kc.dbars + slot, (k / NDESC) & 1u)) break;
    const Stage *st = kc.dring + slot;
    if (st->kind == ST_GEMV) {
      const GemvArgs &a = st->g;
      if (!a.v2) {
        if (k >= done) break;
      } else {
        const V2Plan &pl = kc.pring[slot];
        bool all = true;
        switch (a.fmt) {
          case FMT_BF16: all = stream_gemv<FMT_BF16>(a, pl, kc, smem); break;
          case FMT_INT8: all = stream_gemv<FMT_INT8>(a, pl, kc, smem); break;
          case FMT_Q4_0: all = stream_gemv<FMT_Q4_0>(a, pl, kc, smem); break;
          case FMT_INT4G: all = stream_gemv<FMT_INT4G>(a, pl, kc, smem); break;
        }
        if (!all) break;
      }
    }
    __syncwarp();
    if (lane == 0) {
      kc.pf_seq = k + 1;
      kc.pf_f = 0;
    }
    __syncwarp();
  }
}

// Thread 0, on the way out after an error: wait (bounded) for this CTA's own
// bulk copies still in flight, so none lands after the CTA has exited.
QTB_CALL void drain(KCtx &kc, unsigned cur) {
  constexpr long long LIM = 200000000LL;   // ~0.1 s per copy group
  for (unsigned c = kc.wfill; c != kc.w_issued; c++) mbar_wait(kc.wbars + c % NWSLOT, (c / NWSLOT) & 1u, LIM);
  // page copies: at most the last att_nbuf issued can still be in flight
  const unsigned nb = (unsigned)kc.att_nbuf;
  const unsigned p0 = (kc.att_issued - kc.page_ctr > nb) ? kc.att_issued - nb : kc.page_ctr;
  for (unsigned c = p0; c != kc.att_issued; c++) mbar_wait(kc.bars + c % nb, (c / nb) & 1u, LIM);
  for (unsigned k = cur + 1; k < cur + NDESC && k < kc.n_total; k++)
    mbar_wait(kc.dbars + k % NDESC, (k / NDESC) & 1u, LIM);
  // tcgen05 stages: weight copies in flight, then every MMA issued (one more
  // commit completes after all of them) before the tensor memory is freed
  for (unsigned c = kc.tc_done; c != kc.tc_issued; c++) mbar_wait(kc.tcfull + c % TC_NSLOT, (c / TC_NSLOT) & 1u, LIM);
  for (unsigned g = kc.tc_waited; g != kc.tc_committed; g++) mbar_wait(kc.tcacc + (g & 1u), (g >> 1) & 1u, LIM);
  // single-cluster GEMV stages: the last piece issued into each warp slot
  // (a slot's copies complete in order; a wait skipped after an error does not
  // count as landed)
  if (kc.cl)
    for (int w = 0; w < NWARPS; w++)
      for (unsigned c = kc.cl_iss[w] >= 2u ? kc.cl_iss[w] - 2u : 0u; c < kc.cl_iss[w]; c++)
        mbar_wait(kc.clbars + 2 * w + (c & 1u), (c >> 1) & 1u, LIM);
}

QTB_CALL void argmax_finish(const GemvArgs &a, int B, KCtx &kc);

// Epilogue on final row values val(tl, r, b) held in shared memory
// (s_val[(tl * 16 + r) * sv_ld + b]) for the CTA's tiles t0 .. t0 + nt - 1.
QTB_CALL void v2_epilogue(const GemvArgs &a, int B, int t0, int nt, const float *s_val, int sv_ld, KCtx &kc) {
  const int tid = threadIdx.x;
  auto val = [&](int tl, int r, int b) {
    const int row = 16 * (t0 + tl) + r;
    float v = s_val[(tl * 16 + r) * sv_ld + b];
    if (a.row_scale) v = __ldg(a.row_scale + row) * v;
    if (a.bias) v += __ldg(a.bias + row);
    return v;
  };
  if (a.epi == EPI_STORE || a.epi == EPI_RESID) {
    for (int idx = tid; idx < nt * 16 * B; idx += NTHREADS) {
      const int b = idx % B, r = (idx / B) % 16, tl = idx / (16 * B);
      const int row = 16 * (t0 + tl) + r;
      const float v = val(tl, r, b);
      float *yp = a.y + (size_t)b * a.ldy + row;
      if (a.epi == EPI_RESID) __stcg(yp, __ldcg(yp) + v);
      else __stcg(yp, v);
    }
  } else if (a.epi == EPI_SWIGLU) {
    for (int idx = tid; idx < nt * 8 * B; idx += NTHREADS) {
      const int b = idx % B, pr = (idx / B) % 8, tl = idx / (8 * B);
      const float g = val(tl, 2 * pr, b), u = val(tl, 2 * pr + 1, b);
      const int row = 16 * (t0 + tl) + 2 * pr;
      __stcg(a.y + (size_t)b * a.ldy + (row >> 1), __fdividef(g, 1.0f + expf(-g)) * u);
    }
  } else {  // EPI_ARGMAX
    __shared__ int s_last;
    for (int idx = tid; idx < nt * B; idx += NTHREADS) {
      const int b = idx % B, tl = idx / B;
      unsigned long long best = 0ull;
      for (int r = 0; r < 16; r++) {
        const int row = 16 * (t0 + tl) + r;
        float v = val(tl, r, b);
        if (a.gen) v = codec_logit(a.gen, b, row, v);
        const unsigned long long k = amax_key(v, row);
        best = k > best ? k : best;
      }
      a.amax_ws[(size_t)(t0 + tl) * B + b] = best;
    }
    __syncthreads();
    const int T = a.rows >> 4;
    if (tid == 0) {
      __threadfence();
      const unsigned old = atomicAdd(a.amax_sem, (unsigned)nt);
      s_last = (old + (unsigned)nt == (unsigned)T);
    }
    __syncthreads();
    if (!s_last) return;
    argmax_finish(a, B, kc);
  }
}

// The greedy heads' last step, by the CTA that completed the row tiles'
// per-(16-row tile, batch row) maxima in amax_ws: the code of every batch row
// (first maximum wins: keys order by value, then by lower row), and the next
// input's embedding row gathered from the table.  All threads of the CTA.
QTB_CALL void argmax_finish(const GemvArgs &a, int B, KCtx &kc) {
  {
    const int tid = threadIdx.x;
    const int T = a.rows >> 4;
    __threadfence();
    __shared__ int s_code[64];
    const int warp = tid >> 5, lane = tid & 31;
    for (int b = warp; b < B; b += NWARPS) {
      unsigned long long best = 0ull;
      for (int tt = lane; tt < T; tt += 32) {
        const unsigned long long k = __ldcg(a.amax_ws + (size_t)tt * B + b);
        best = k > best ? k : best;
      }
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) {
        const unsigned long long o = shfl_xor_u64(best, m);
        best = o > best ? o : best;
      }
      int code = (int)(0xffffffffu - (unsigned)(best & 0xffffffffull));
      // a running slot with a temperature samples instead of taking the maximum
      if (a.gen && a.gen->enabled && a.gen->sampling && !__ldcg(a.gen->done + b) && __ldcg(a.gen->temp + b) >= 1e-6f)
        code = sample_codec(a.gen, b);
      if (lane == 0) {
        if (a.gen && a.gen->enabled && !__ldcg(a.gen->done + b)) {
          // the codec head of a running slot: EOS stops it; other codes count
          // towards its repetition penalty
          if (code == a.gen->eos_row) {
            code = a.gen->eos_token;
            a.gen->done[b] = 1;
          } else {
            a.gen->rep_count[(size_t)b * a.gen->vocab + code] += 1;
          }
        }
        a.codes[(size_t)b * a.code_stride] = code;
        s_code[b] = code;
      }
    }
    __syncthreads();
    if (a.emb_table) {
      for (int idx = tid; idx < B * (a.emb_ld / 8); idx += NTHREADS) {
        const int b = idx / (a.emb_ld / 8), i = (idx % (a.emb_ld / 8)) * 8;
        int cb = s_code[b];
        if (cb < 0 || cb >= a.emb_rows) { if (i == 0) raise_err(kc, ERR_BAD_CODE, cb); cb = 0; }
        const uint4 v = ld_nc_u4(a.emb_table + (size_t)cb * a.emb_ld + i);
        float *dst = a.emb_out + (size_t)b * a.emb_out_ld + i;
        __stcg(reinterpret_cast<float4 *>(dst), make_float4(bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y)));
        __stcg(reinterpret_cast<float4 *>(dst + 4), make_float4(bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w)));
      }
    }
    if (tid == 0) *a.amax_sem = 0u;
  }
}

template <int FMT, int NCH, int P>
__device__ __noinline__ void gemv2_stage_t(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  using Tr = FmtTraits<FMT>;
  constexpr bool F16 = (FMT != FMT_BF16);
  constexpr bool XSUM = (FMT == FMT_Q4_0 || FMT == FMT_INT4G);
  const V2Sched s = v2_sched<FMT>(a, kc.pring[kc.seq % NDESC]);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
  const int ent = 4 * min(8, P * B);
  const int xsum_n = a.K >> 5;
  float *s_inv = reinterpret_cast<float *>(smem + SM_R_OFF);
  float *s_red = s_inv + 64;   // [nt][NWARPS][16][B]
  float *s_xsum = reinterpret_cast<float *>(smem + SM_X_OFF);
  const int xsum_floats = XSUM ? ((B * xsum_n + 3) & ~3) : 0;
  uint2 *s_xf = reinterpret_cast<uint2 *>(s_xsum + xsum_floats);

  // this stage's first fills, unless the streamer issued them already
  ckpt(kc, 11);
  if (warp == 0 && kc.pf_seq <= kc.seq) stream(kc, smem, kc.seq, kc.seq + 1);
  ckpt(kc, 0);
  if (s.nt == 0) return;

  {
    const int mq = (B * (a.K >> 2) + NTHREADS - 1) / NTHREADS;
    if (mq <= 1) stage_x_fused<F16, P, 1>(a, B, ent, s_inv, s_xsum, s_xf, XSUM, kc, smem);
    else if (mq <= 2) stage_x_fused<F16, P, 2>(a, B, ent, s_inv, s_xsum, s_xf, XSUM, kc, smem);
    else if (mq <= 4) stage_x_fused<F16, P, 4>(a, B, ent, s_inv, s_xsum, s_xf, XSUM, kc, smem);
    else stage_x_fused<F16, P, 8>(a, B, ent, s_inv, s_xsum, s_xf, XSUM, kc, smem);
  }
  for (int i = tid; i < s.nt * NWARPS * 16 * B; i += NTHREADS) s_red[i] = 0.f;
  __syncthreads();
  ckpt(kc, 2);

  constexpr int CPS = WSLOT_BYTES / (512 + 8 * Tr::GSZ);   // chunks per ring slot (== s.cps)
  const int per_wave = NWSLOT * CPS;
  const unsigned wf = kc.wfill;
  for (int w0 = 0; w0 < s.L; w0 += per_wave) {
    // Warps take equal runs of whole 4-chunk groups (tile lengths, wave
    // lengths and tile starts are multiples of 4 chunks).
    const int wl = min(per_wave, s.L - w0);
    const int q4 = (wl + 3) >> 2;
    const int cb = w0 + 4 * ((warp * q4) / NWARPS);
    const int ce = min(w0 + wl, w0 + 4 * (((warp + 1) * q4) / NWARPS));
    // four accumulator sets: the MMAs of a 4-chunk group are independent
    float acc[NCH][4], acc1[NCH][4], acc2[NCH][4], acc3[NCH][4], res[NCH][2];
#pragma unroll
    for (int j = 0; j < NCH; j++)
#pragma unroll
      for (int e2 = 0; e2 < 4; e2++) { acc[j][e2] = acc1[j][e2] = acc2[j][e2] = acc3[j][e2] = 0.f; res[j][e2 & 1] = 0.f; }
    auto flush = [&](int tl) {
#pragma unroll
      for (int j = 0; j < NCH; j++)
#pragma unroll
        for (int e2 = 0; e2 < 4; e2++) {
          acc[j][e2] = (acc[j][e2] + acc1[j][e2]) + (acc2[j][e2] + acc3[j][e2]);
          acc1[j][e2] = acc2[j][e2] = acc3[j][e2] = 0.f;
        }
      acc_finish<FMT, NCH, P>(acc, res);
#pragma unroll
      for (int j = 0; j < NCH; j++) {
        const int b = col_batch<P>(j, tig);
        if (b < B && col_owner<P>(tig)) {
          s_red[((tl * NWARPS + warp) * 16 + gid) * B + b] += res[j][0];
          s_red[((tl * NWARPS + warp) * 16 + gid + 8) * B + b] += res[j][1];
        }
        acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        res[j][0] = res[j][1] = 0.f;
      }
    };
    auto load = [&](int ci, uint4 &wv, uint4 &gv) {
      const int f = ci / CPS, o = ci - f * CPS;
      const char *slot = smem + SM_W_OFF + ((wf + (unsigned)f) % NWSLOT) * WSLOT_BYTES;
      wv = *reinterpret_cast<const uint4 *>(slot + o * 512 + lane * 16);
      gv = make_uint4(0u, 0u, 0u, 0u);
      if (Tr::GSZ == 8) {
        const uint2 g = *reinterpret_cast<const uint2 *>(slot + CPS * 512 + o * 64 + gid * 8);
        gv = make_uint4(g.x, g.y, 0u, 0u);
      } else if (Tr::GSZ == 16) {
        gv = *reinterpret_cast<const uint4 *>(slot + CPS * 512 + o * 128 + gid * 16);
      }
    };
    // the fills this warp reads (after a failed wait the CTA only runs out the stage)
    if (cb < ce) {
      for (int f = cb / CPS; f <= (ce - 1) / CPS; f++) {
        const unsigned ctr = wf + (unsigned)f;
        if (!kc.local_err && !mbar_wait(kc.wbars + (ctr % NWSLOT), (ctr / NWSLOT) & 1u, WAIT_LIMIT_CYCLES))
          raise_err(kc, ERR_MBAR_TIMEOUT, f);
      }
    }
    ckpt(kc, 9);   // warp 0's weights ready
    int ci = cb;
    while (ci < ce) {
      const int tl = ci / s.kc;
      const int te = min(ce, (tl + 1) * s.kc);
      const int c0 = s.kb - tl * s.kc;   // chunk ci is column chunk c0 + ci of its tile
      for (; ci + 4 <= te; ci += 4) {
        uint4 wv[4], gv[4];
#pragma unroll
        for (int u = 0; u < 4; u++) load(ci + u, wv[u], gv[u]);
#pragma unroll
        for (int u = 0; u < 4; u++) {
          if (u & 1) mma_chunk<FMT, NCH>(wv[u], gv[u], c0 + ci + u, s_xf, ent, s_xsum, xsum_n, B, acc2, res, acc3);
          else mma_chunk<FMT, NCH>(wv[u], gv[u], c0 + ci + u, s_xf, ent, s_xsum, xsum_n, B, acc, res, acc1);
        }
      }
      for (; ci < te; ci++) {
        uint4 wv, gv;
        load(ci, wv, gv);
        mma_chunk<FMT, NCH>(wv, gv, c0 + ci, s_xf, ent, s_xsum, xsum_n, B, acc, res, acc1);
      }
      flush(tl);
    }
    ckpt(kc, 10);   // warp 0 done with its chunks
    ckpt_w(kc, 24);
    __syncthreads();
    if (w0 + per_wave < s.L && warp == 0) {   // this wave's slots are free again
      if (lane == 0) kc.w_free = kc.wfill + (unsigned)((w0 + per_wave) / CPS);
      __syncwarp();
      stream(kc, smem, kc.seq, kc.seq + 2);
    }
  }
  if (tid == 0) {   // every warp is past its last slot read
    kc.wfill += (unsigned)s.nfill;
    kc.w_free = kc.wfill;
  }
  ckpt(kc, 3);

  // per tile: sum the warps' partials in warp order -> s_val[tl][16][B]
  float *s_val = s_red + s.nt * NWARPS * 16 * B;
  for (int idx = tid; idx < s.nt * 16 * B; idx += NTHREADS) {
    const int b = idx % B, r = (idx / B) % 16, tl2 = idx / (16 * B);
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NWARPS; w++) v += s_red[((tl2 * NWARPS + w) * 16 + r) * B + b];
    s_val[idx] = v;
  }
  __syncthreads();
  ckpt(kc, 4);
  v2_epilogue(a, B, s.t0, s.nt, s_val, B, kc);
  ckpt(kc, 5);
}

// ------------------------------------------ small-batch int8: s8 tensor cores
//
// The activation (after the fused RMSNorm) is carried as four signed 8-bit
// parts per value, x = sx * (a0 + a1 / 2^7 + a2 / 2^14 + a3 / 2^21), sx =
// max|x| / 127 per batch row (the fixed-point value rint(x / sx * 2^21) split
// into a leading part and three balanced base-128 digits), which represents x
// to ~2^-29 of max|x|.  The int8
// weights then feed the integer MMA (m16n8k32, s8 x s8 -> s32, exact) as they
// are stored: no per-weight conversion instructions at all.  The parts of batch
// row b are MMA columns 4b .. 4b+3; per k32 chunk c and column chunk j the
// staged activation holds one (b0, b1) register pair per lane.
template <int MAXQ>
// Stages columns [k0, k0 + K) of the activation (a piece of it for a split
// stage; then the part scale is the piece's own); chunk c of the staged
// range is column chunk k0/32 + c.
__device__ __noinline__ void stage_x_s8(const GemvArgs &a, int B, int nch, int k0, int K, float *s_scl,
                                        uint32_t *s_xw, float *s_zero, int n_zero, KCtx &kc) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nk4 = K >> 2;
  const int nq = B * nk4;
  float v[MAXQ][4], g[MAXQ][4];
  float ss[4] = {0.f, 0.f, 0.f, 0.f}, mx[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < MAXQ; i++) {
    const int t = tid + i * NTHREADS;
    if (t < nq) {
      const int b = t / nk4, k = 4 * (t - b * nk4);
      const float4 x4 = __ldcg(reinterpret_cast<const float4 *>(a.x + (size_t)b * a.ldx + k0 + k));
      v[i][0] = x4.x; v[i][1] = x4.y; v[i][2] = x4.z; v[i][3] = x4.w;
      if (a.norm_w) {
        const float4 g4 = __ldg(reinterpret_cast<const float4 *>(a.norm_w + k0 + k));
        g[i][0] = g4.x; g[i][1] = g4.y; g[i][2] = g4.z; g[i][3] = g4.w;
      } else {
        g[i][0] = g[i][1] = g[i][2] = g[i][3] = 1.f;
      }
    }
  }
  __shared__ float s_red2[NWARPS][8];
#pragma unroll
  for (int i = 0; i < MAXQ; i++) {
    const int t = tid + i * NTHREADS;
    if (t < nq) {
      const int b = t / nk4;
      float s2 = 0.f, m2 = 0.f;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        s2 += v[i][e] * v[i][e];
        m2 = fmaxf(m2, fabsf(v[i][e] * g[i][e]));
      }
#pragma unroll
      for (int bb = 0; bb < 4; bb++)
        if (b == bb) { ss[bb] += s2; mx[bb] = fmaxf(mx[bb], m2); }
    }
  }
  ckpt(kc, 8);
  ckpt_w(kc, 16);
#pragma unroll
  for (int bb = 0; bb < 4; bb++) {
    if (bb < B) {   // warp-uniform
      const float w = warp_sum(ss[bb]), m = warp_max(mx[bb]);
      if (lane == 0) { s_red2[warp][bb] = w; s_red2[warp][4 + bb] = m; }
    }
  }
  for (int i = tid; i < n_zero; i += NTHREADS) s_zero[i] = 0.f;   // the caller's partial sums
  ckpt(kc, 12);
  __syncthreads();
  ckpt(kc, 13);
  // every thread derives the scales itself (broadcast reads): no second barrier
  float inv[4], rsx[4];
#pragma unroll
  for (int bb = 0; bb < 4; bb++) {
    inv[bb] = 1.f; rsx[bb] = 1.f;
    if (bb < B) {
      float tot = 0.f, m = 0.f;
#pragma unroll
      for (int w = 0; w < NWARPS; w++) { tot += s_red2[w][bb]; m = fmaxf(m, s_red2[w][4 + bb]); }
      // (hardware reciprocal square root: within 2 ulp of the reference's
      // 1 / sqrtf, far inside the path's tolerance, and off the IEEE slow path)
      inv[bb] = a.norm_w ? rsqrtf(tot * __frcp_rn((float)K) + a.eps) : 1.0f;
      const float sx = fmaxf(m * inv[bb], 1e-30f) * (1.0f / 127.0f);
      rsx[bb] = __frcp_rn(sx);
      if (tid == 0) s_scl[4 + bb] = sx;   // part scale, read after the caller's barrier
    }
  }
  ckpt(kc, 14);
#pragma unroll
  for (int i = 0; i < MAXQ; i++) {
    const int t = tid + i * NTHREADS;
    if (t < nq) {
      const int b = t / nk4, k = 4 * (t - b * nk4);
      float iv = inv[0], rs = rsx[0];
#pragma unroll
      for (int bb = 1; bb < 4; bb++)
        if (b == bb) { iv = inv[bb]; rs = rsx[bb]; }
      uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float xn = a.norm_w ? (v[i][e] * iv) * g[i][e] : v[i][e];
        const float r = fminf(fmaxf(xn * rs, -127.f), 127.f);
        // fixed point I = r * 2^21, then balanced base-128 digits:
        // I = a0 2^21 + d1 2^14 + d2 2^7 + d3, |d| <= 64, |a0| <= 127
        int I = __float2int_rn(r * 2097152.f);
        const int d3 = ((I + 64) & 127) - 64;
        I = (I - d3) >> 7;
        const int d2 = ((I + 64) & 127) - 64;
        I = (I - d2) >> 7;
        const int d1 = ((I + 64) & 127) - 64;
        const int a0 = (I - d1) >> 7;
        w[0] |= ((uint32_t)a0 & 0xffu) << (8 * e);
        w[1] |= ((uint32_t)d1 & 0xffu) << (8 * e);
        w[2] |= ((uint32_t)d2 & 0xffu) << (8 * e);
        w[3] |= ((uint32_t)d3 & 0xffu) << (8 * e);
      }
      const int c = k >> 5, half = (k >> 4) & 1, tq = (k >> 2) & 3;
#pragma unroll
      for (int p = 0; p < 4; p++) {
        const int col = 4 * b + p, j = col >> 3, gid = col & 7;
        s_xw[(((c * nch + j) * 32) + gid * 4 + tq) * 2 + half] = w[p];
      }
    }
  }
  ckpt(kc, 15);
}

// The two halves of a split stage (2-CTA cluster): the second half stores its
// per-row sums into the first half's shared memory and arrives on its
// mbarrier; the first half waits (bounded), adds them to its own (own first:
// fixed order) and returns true to run the epilogue.
QTB_CALL bool pair_combine(float *s_val, int n, int role, char *smem, KCtx &kc) {
  float *recv = reinterpret_cast<float *>(smem + SM_PAIR_OFF);
  const int tid = threadIdx.x;
  if (role == 2) {
    for (int i = tid; i < n; i += NTHREADS) st_cluster_f32(cluster_map(recv + i, 0), s_val[i]);
    __syncthreads();
    if (tid == 0) mbar_arrive_remote(cluster_map(kc.pbar, 0));
    return false;
  }
  if (!mbar_wait_cluster(kc.pbar, kc.pair_ctr & 1u, WAIT_LIMIT_CYCLES)) {
    if (tid == 0) raise_err(kc, ERR_MBAR_TIMEOUT, -4);
  }
  for (int i = tid; i < n; i += NTHREADS) s_val[i] = s_val[i] + recv[i];
  __syncthreads();
  if (tid == 0) kc.pair_ctr++;
  return true;
}

template <int NCH>
__device__ __noinline__ void gemv2_s8_t(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  const V2Sched s = v2_sched<FMT_INT8>(a, kc.pring[kc.seq % NDESC]);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
  float *s_scl = reinterpret_cast<float *>(smem + SM_R_OFF);
  float *s_red = s_scl + 64;   // [nt][NWARPS][16][B]
  uint32_t *s_xw = reinterpret_cast<uint32_t *>(smem + SM_X_OFF);
  const uint2 *s_xf = reinterpret_cast<const uint2 *>(s_xw);

  ckpt(kc, 11);
  if (warp == 0 && kc.pf_seq <= kc.seq) stream(kc, smem, kc.seq, kc.seq + 1);   // this stage's first fills, if not issued yet
  ckpt(kc, 0);
  if (s.nt == 0) return;
  // STORE / RESID with one output per thread: load the row scale and the
  // residual now, so the epilogue does not wait on L2 after the MMA
  const int role = kc.pring[kc.seq % NDESC].pair;
  const bool fast_epi = (a.epi == EPI_STORE || a.epi == EPI_RESID) && !a.bias && s.nt * 16 * B <= NTHREADS &&
                        role != 2;
  float pre_rs = 1.f, pre_res = 0.f;
  if (fast_epi && tid < s.nt * 16 * B) {
    const int b = tid % B, r = (tid / B) % 16, tl = tid / (16 * B);
    const int row = 16 * (s.t0 + tl) + r;
    if (a.row_scale) pre_rs = __ldg(a.row_scale + row);
    if (a.epi == EPI_RESID) pre_res = __ldcg(a.y + (size_t)b * a.ldy + row);
  }
  {
    const int mq = (B * (32 * s.kc >> 2) + NTHREADS - 1) / NTHREADS;
    const int nz = s.nt * NWARPS * 16 * B;
    const int k0 = 32 * s.kb, Kp = 32 * s.kc;   // the staged columns (a piece for split stages)
    if (mq <= 1) stage_x_s8<1>(a, B, NCH, k0, Kp, s_scl, s_xw, s_red, nz, kc);
    else if (mq <= 2) stage_x_s8<2>(a, B, NCH, k0, Kp, s_scl, s_xw, s_red, nz, kc);
    else if (mq <= 4) stage_x_s8<4>(a, B, NCH, k0, Kp, s_scl, s_xw, s_red, nz, kc);
    else stage_x_s8<8>(a, B, NCH, k0, Kp, s_scl, s_xw, s_red, nz, kc);
  }
  __syncthreads();
  ckpt(kc, 2);

  constexpr int CPS = WSLOT_BYTES / 512;
  const int per_wave = NWSLOT * CPS;
  const unsigned wf = kc.wfill;
  // column pair (2 tig, 2 tig + 1) of chunk j = parts (2 (tig & 1), +1) of
  // batch row 2 j + tig / 2
  const float wlo = (tig & 1) ? (1.0f / 16384.0f) : 1.0f, whi = (tig & 1) ? (1.0f / 2097152.0f) : (1.0f / 128.0f);
  for (int w0 = 0; w0 < s.L; w0 += per_wave) {
    const int wl = min(per_wave, s.L - w0);
    const int q4 = (wl + 3) >> 2;
    const int cb = w0 + 4 * ((warp * q4) / NWARPS);
    const int ce = min(w0 + wl, w0 + 4 * (((warp + 1) * q4) / NWARPS));
    int acc[4][NCH][4];
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int j = 0; j < NCH; j++) acc[u][j][0] = acc[u][j][1] = acc[u][j][2] = acc[u][j][3] = 0;
    auto flush = [&](int tl) {
#pragma unroll
      for (int j = 0; j < NCH; j++) {
        const int i0 = acc[0][j][0] + acc[1][j][0] + acc[2][j][0] + acc[3][j][0];
        const int i1 = acc[0][j][1] + acc[1][j][1] + acc[2][j][1] + acc[3][j][1];
        const int i2 = acc[0][j][2] + acc[1][j][2] + acc[2][j][2] + acc[3][j][2];
        const int i3 = acc[0][j][3] + acc[1][j][3] + acc[2][j][3] + acc[3][j][3];
        float r0 = (float)i0 * wlo + (float)i1 * whi;   // row gid
        float r1 = (float)i2 * wlo + (float)i3 * whi;   // row gid + 8
        r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
        r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
        const int b = 2 * j + (tig >> 1);
        if ((tig & 1) == 0 && b < B) {
          const float sx = s_scl[4 + b];
          s_red[((tl * NWARPS + warp) * 16 + gid) * B + b] += r0 * sx;
          s_red[((tl * NWARPS + warp) * 16 + gid + 8) * B + b] += r1 * sx;
        }
#pragma unroll
        for (int u = 0; u < 4; u++) acc[u][j][0] = acc[u][j][1] = acc[u][j][2] = acc[u][j][3] = 0;
      }
    };
    auto load = [&](int ci) -> uint4 {
      const int f = ci / CPS, o = ci - f * CPS;
      const char *slot = smem + SM_W_OFF + ((wf + (unsigned)f) % NWSLOT) * WSLOT_BYTES;
      return *reinterpret_cast<const uint4 *>(slot + o * 512 + lane * 16);
    };
    if (cb < ce) {   // the fills this warp reads (after a failed wait the CTA only runs out the stage)
      for (int f = cb / CPS; f <= (ce - 1) / CPS; f++) {
        const unsigned ctr = wf + (unsigned)f;
        if (!kc.local_err && !mbar_wait(kc.wbars + (ctr % NWSLOT), (ctr / NWSLOT) & 1u, WAIT_LIMIT_CYCLES))
          raise_err(kc, ERR_MBAR_TIMEOUT, f);
      }
    }
    ckpt(kc, 9);
    int ci = cb;
    while (ci < ce) {
      const int tl = ci / s.kc;
      const int te = min(ce, (tl + 1) * s.kc);
      const int c0 = -tl * s.kc;   // staged chunk of chunk ci
      for (; ci + 4 <= te; ci += 4) {
        uint4 wv[4];
#pragma unroll
        for (int u = 0; u < 4; u++) wv[u] = load(ci + u);
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
          for (int j = 0; j < NCH; j++) {
            const uint2 bx = s_xf[((c0 + ci + u) * NCH + j) * 32 + lane];
            mma_s8(acc[u][j], wv[u], bx.x, bx.y);
          }
      }
      for (; ci < te; ci++) {
        const uint4 wv = load(ci);
#pragma unroll
        for (int j = 0; j < NCH; j++) {
          const uint2 bx = s_xf[((c0 + ci) * NCH + j) * 32 + lane];
          mma_s8(acc[0][j], wv, bx.x, bx.y);
        }
      }
      flush(tl);
    }
    ckpt(kc, 10);
    __syncthreads();
    if (w0 + per_wave < s.L && warp == 0) {   // this wave's slots are free again
      if (lane == 0) kc.w_free = kc.wfill + (unsigned)((w0 + per_wave) / CPS);
      __syncwarp();
      stream(kc, smem, kc.seq, kc.seq + 2);
    }
  }
  if (tid == 0) {
    kc.wfill += (unsigned)s.nfill;
    kc.w_free = kc.wfill;
  }
  ckpt(kc, 3);
  float *s_val = s_red + s.nt * NWARPS * 16 * B;
  for (int idx = tid; idx < s.nt * 16 * B; idx += NTHREADS) {
    const int b = idx % B, r = (idx / B) % 16, tl2 = idx / (16 * B);
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NWARPS; w++) v += s_red[((tl2 * NWARPS + w) * 16 + r) * B + b];
    s_val[idx] = v;
  }
  __syncthreads();
  ckpt(kc, 4);
  if (role && !pair_combine(s_val, 16 * B, role, smem, kc)) return;
  ckpt(kc, 24);
  if (fast_epi) {
    if (tid < s.nt * 16 * B) {
      const int b = tid % B, r = (tid / B) % 16, tl = tid / (16 * B);
      const int row = 16 * (s.t0 + tl) + r;
      __stcg(a.y + (size_t)b * a.ldy + row, pre_res + pre_rs * s_val[tid]);
    }
  } else {
    v2_epilogue(a, B, s.t0, s.nt, s_val, B, kc);
  }
  ckpt(kc, 5);
}

// ====================================== GEMV stage, single-cluster schedule =
//
// Small batches (B <= 4) when the launch is one cluster of CL_G CTAs.  A CTA
// owns whole 16-row tiles t0 .. t0 + nt - 1; with fewer tiles than warps each
// tile's K is cut into ks slices (a power of two) so every warp has a unit
// (tile, slice) of kc = nck / ks chunks; warp w takes units w, w + 8, ...
// Each warp streams its own units' weights, in pieces of up to cl_pc chunks,
// through its two slots of the weight-ring region (one piece computing while
// the next is in flight), and issues the first two pieces of the next GEMV
// stage before the cluster barrier, so the weight stream does not stop at
// stage boundaries.  The activation is staged as in the other small-batch
// stages; each unit's 16 rows go to shared memory and the CTA adds a tile's
// slices in slice order (deterministic) before the common epilogue.
//
// Host plan (V2Plan): t0, nt, kb = ks, kc = chunks per unit, L = pieces per
// unit, the rest zero.
template <int FMT>
QTB_HOST_DEV constexpr int cl_pc() { return CL_SLOT_BYTES / (512 + 8 * FmtTraits<FMT>::GSZ); }
QTB_HOST_DEV int cl_pc_fmt(int fmt) {
  return fmt == FMT_BF16 ? cl_pc<FMT_BF16>() : fmt == FMT_INT8 ? cl_pc<FMT_INT8>()
       : fmt == FMT_Q4_0 ? cl_pc<FMT_Q4_0>() : cl_pc<FMT_INT4G>();
}

QTB_HOST_DEV V2Plan cl_plan(int fmt, int rows, int K, int cta, int G) {
  const int ck = fmt == FMT_BF16 ? 1 : (fmt == FMT_INT8 ? 2 : 4);
  const int T = rows >> 4, nck = K / (16 * ck);
  V2Plan p;
  p.t0 = (int)((long long)cta * T / G);
  p.nt = (int)((long long)(cta + 1) * T / G) - p.t0;
  int ks = 1;
  while (p.nt > 0 && 2 * ks * p.nt <= NWARPS && nck % (2 * ks) == 0 && nck / (2 * ks) >= 4) ks *= 2;
  p.kb = ks;
  p.kc = nck / ks;
  const int pc = cl_pc_fmt(fmt);
  p.L = (p.kc + pc - 1) / pc;
  p.nfill = 0;
  p.pair = 0;
  p.pad = 0;
  return p;
}

struct ClPiece { int tl, s, c0, n; };   // local tile, slice, first chunk in the tile, chunks

QTB_DEV int cl_npieces(const V2Plan &p, int w) {
  const int units = p.nt * p.kb;
  return w < units ? ((units - 1 - w) / NWARPS + 1) * p.L : 0;
}
QTB_DEV ClPiece cl_piece(const V2Plan &p, int pc, int w, int q) {
  const int j = q / p.L, pp = q - j * p.L, u = w + NWARPS * j;
  ClPiece r;
  r.tl = u / p.kb;
  r.s = u - r.tl * p.kb;
  r.c0 = r.s * p.kc + pp * pc;
  r.n = min(pc, p.kc - pp * pc);
  return r;
}

// Lane 0 of warp w: bulk-copy piece q of the warp's units of stage (a, p)
// into the warp's next slot.
template <int FMT>
QTB_DEV void cl_issue(const GemvArgs &a, const V2Plan &p, int w, int q, KCtx &kc, char *smem) {
  using Tr = FmtTraits<FMT>;
  constexpr int PC = cl_pc<FMT>();
  const ClPiece pc = cl_piece(p, PC, w, q);
  const size_t base = (size_t)(p.t0 + pc.tl) * (p.kb * p.kc) + pc.c0;
  const unsigned k = kc.cl_iss[w];
  char *dst = smem + SM_W_OFF + (2 * w + (int)(k & 1u)) * CL_SLOT_BYTES;
  uint64_t *bar = kc.clbars + 2 * w + (k & 1u);
  const uint32_t wb = (uint32_t)pc.n * 512u, gb = (uint32_t)pc.n * 8u * Tr::GSZ;
  const uint64_t pol = a.evict_last ? kc.pol_last : kc.pol_first;
  fence_proxy_async_smem();   // the slot was last read through the generic proxy
  mbar_arrive_expect_tx(bar, wb + gb);
  bulk_g2s_hint(dst, a.w + base * 512, wb, bar, pol);
  if (Tr::GSZ) bulk_g2s_hint(dst + PC * 512, a.gsz + base * (8 * Tr::GSZ), gb, bar, pol);
  kc.cl_iss[w] = k + 1u;
}

// Lane 0 of warp w, after its last piece of the current stage: the first two
// pieces of the next GEMV stage within the landed descriptors.
QTB_DEV void cl_issue_ahead(KCtx &kc, char *smem, int w) {
  if (kc.local_err) return;
  for (unsigned k = kc.seq + 1; k < kc.n_total && k <= kc.seq + STREAM_AHEAD; k++) {
    const int slot = (int)(k % NDESC);
    if (!mbar_test(kc.dbars + slot, (k / NDESC) & 1u)) return;
    const Stage *st = kc.dring + slot;
    if (st->kind != ST_GEMV) continue;
    if (!st->g.cl) return;
    const V2Plan &p = kc.pring[slot];
    const int n = min(2, cl_npieces(p, w));
    for (int q = 0; q < n; q++) {
      switch (st->g.fmt) {
        case FMT_BF16: cl_issue<FMT_BF16>(st->g, p, w, q, kc, smem); break;
        case FMT_INT8: cl_issue<FMT_INT8>(st->g, p, w, q, kc, smem); break;
        case FMT_Q4_0: cl_issue<FMT_Q4_0>(st->g, p, w, q, kc, smem); break;
        default: cl_issue<FMT_INT4G>(st->g, p, w, q, kc, smem); break;
      }
    }
    kc.cl_pre[w] = k;
    return;
  }
}

// Lane 0 of warp w at the start of a stage: its first pieces, unless issued
// ahead by the previous GEMV stage.
template <int FMT>
QTB_DEV void cl_start(const GemvArgs &a, const V2Plan &p, int w, int np, KCtx &kc, char *smem) {
  const int have = (kc.cl_pre[w] == kc.seq) ? (int)(kc.cl_iss[w] - kc.cl_q[w]) : 0;
  if (kc.local_err) return;
  for (int q = have; q < min(2, np); q++) cl_issue<FMT>(a, p, w, q, kc, smem);
}

// Every lane of the warp: wait for the warp's next piece (bounded); returns its slot.
QTB_DEV const char *cl_wait(KCtx &kc, char *smem, int w, int q) {
  const unsigned k = kc.cl_q[w];
  if (!kc.local_err && !mbar_wait(kc.clbars + 2 * w + (k & 1u), (k >> 1) & 1u, WAIT_LIMIT_CYCLES))
    raise_err(kc, ERR_MBAR_TIMEOUT, 4000 + q);
  return smem + SM_W_OFF + (2 * w + (int)(k & 1u)) * CL_SLOT_BYTES;
}
// ... and after reading it: release the slot, refill it with piece q + 2.
template <int FMT>
QTB_DEV void cl_release(const GemvArgs &a, const V2Plan &p, int w, int q, int np, KCtx &kc, char *smem) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    kc.cl_q[w] += 1u;
    // after an error no new copy goes out (the ones in flight are drained)
    if (q + 2 < np && !kc.local_err) cl_issue<FMT>(a, p, w, q + 2, kc, smem);
  }
  __syncwarp();
}

// bf16 / q4_0 / int4 g32 weights (f16 / bf16 MMA on the staged parts).
template <int FMT, int NCH, int P>
__device__ __noinline__ void gemv_cl_t(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  using Tr = FmtTraits<FMT>;
  constexpr bool F16 = (FMT != FMT_BF16);
  constexpr bool XSUM = (FMT == FMT_Q4_0 || FMT == FMT_INT4G);
  constexpr int PC = cl_pc<FMT>();
  const V2Plan p = kc.pring[kc.seq % NDESC];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
  const int ent = 4 * min(8, P * B);
  const int xsum_n = a.K >> 5;
  float *s_inv = reinterpret_cast<float *>(smem + SM_R_OFF);
  float *s_red = s_inv + 64;   // [nt * ks][16][B]
  float *s_xsum = reinterpret_cast<float *>(smem + SM_X_OFF);
  const int xsum_floats = XSUM ? ((B * xsum_n + 3) & ~3) : 0;
  uint2 *s_xf = reinterpret_cast<uint2 *>(s_xsum + xsum_floats);
  const int np = cl_npieces(p, warp);

  ckpt(kc, 11);
  if (lane == 0) cl_start<FMT>(a, p, warp, np, kc, smem);
  __syncwarp();
  ckpt(kc, 0);
  if (p.nt == 0) return;
  {
    const int mq = (B * (a.K >> 2) + NTHREADS - 1) / NTHREADS;
    if (mq <= 1) stage_x_fused<F16, P, 1>(a, B, ent, s_inv, s_xsum, s_xf, XSUM, kc, smem);
    else if (mq <= 2) stage_x_fused<F16, P, 2>(a, B, ent, s_inv, s_xsum, s_xf, XSUM, kc, smem);
    else if (mq <= 4) stage_x_fused<F16, P, 4>(a, B, ent, s_inv, s_xsum, s_xf, XSUM, kc, smem);
    else stage_x_fused<F16, P, 8>(a, B, ent, s_inv, s_xsum, s_xf, XSUM, kc, smem);
  }
  __syncthreads();
  ckpt(kc, 2);

  float acc[NCH][4], acc1[NCH][4], acc2[NCH][4], acc3[NCH][4], res[NCH][2];
#pragma unroll
  for (int j = 0; j < NCH; j++)
#pragma unroll
    for (int e2 = 0; e2 < 4; e2++) { acc[j][e2] = acc1[j][e2] = acc2[j][e2] = acc3[j][e2] = 0.f; res[j][e2 & 1] = 0.f; }
  for (int q = 0; q < np; q++) {
    const ClPiece pc = cl_piece(p, PC, warp, q);
    const char *slot = cl_wait(kc, smem, warp, q);
    if (q == 0) ckpt(kc, 12);
    auto load = [&](int i, uint4 &wv, uint4 &gv) {
      wv = *reinterpret_cast<const uint4 *>(slot + i * 512 + lane * 16);
      gv = make_uint4(0u, 0u, 0u, 0u);
      if (Tr::GSZ == 8) {
        const uint2 g = *reinterpret_cast<const uint2 *>(slot + PC * 512 + i * 64 + gid * 8);
        gv = make_uint4(g.x, g.y, 0u, 0u);
      } else if (Tr::GSZ == 16) {
        gv = *reinterpret_cast<const uint4 *>(slot + PC * 512 + i * 128 + gid * 16);
      }
    };
    int i = 0;
    for (; i + 4 <= pc.n; i += 4) {
      uint4 wv[4], gv[4];
#pragma unroll
      for (int u = 0; u < 4; u++) load(i + u, wv[u], gv[u]);
#pragma unroll
      for (int u = 0; u < 4; u++) {
        if (u & 1) mma_chunk<FMT, NCH>(wv[u], gv[u], pc.c0 + i + u, s_xf, ent, s_xsum, xsum_n, B, acc2, res, acc3);
        else mma_chunk<FMT, NCH>(wv[u], gv[u], pc.c0 + i + u, s_xf, ent, s_xsum, xsum_n, B, acc, res, acc1);
      }
    }
    for (; i < pc.n; i++) {
      uint4 wv, gv;
      load(i, wv, gv);
      mma_chunk<FMT, NCH>(wv, gv, pc.c0 + i, s_xf, ent, s_xsum, xsum_n, B, acc, res, acc1);
    }
    cl_release<FMT>(a, p, warp, q, np, kc, smem);
    if (pc.c0 + pc.n == (pc.s + 1) * p.kc) {   // the unit's last piece: its 16 rows out
#pragma unroll
      for (int j = 0; j < NCH; j++)
#pragma unroll
        for (int e2 = 0; e2 < 4; e2++) {
          acc[j][e2] = (acc[j][e2] + acc1[j][e2]) + (acc2[j][e2] + acc3[j][e2]);
          acc1[j][e2] = acc2[j][e2] = acc3[j][e2] = 0.f;
        }
      acc_finish<FMT, NCH, P>(acc, res);
      const int u = pc.tl * p.kb + pc.s;
#pragma unroll
      for (int j = 0; j < NCH; j++) {
        const int b = col_batch<P>(j, tig);
        if (b < B && col_owner<P>(tig)) {
          s_red[(u * 16 + gid) * B + b] = res[j][0];
          s_red[(u * 16 + gid + 8) * B + b] = res[j][1];
        }
        acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        res[j][0] = res[j][1] = 0.f;
      }
    }
  }
  ckpt_w(kc, 24);
  if (lane == 0) cl_issue_ahead(kc, smem, warp);
  __syncthreads();
  ckpt(kc, 3);
  float *s_val = s_red;
  if (p.kb > 1) {   // a tile's slices, in slice order
    s_val = s_red + p.nt * p.kb * 16 * B;
    for (int idx = tid; idx < p.nt * 16 * B; idx += NTHREADS) {
      const int rb = idx % (16 * B), tl = idx / (16 * B);
      float v = 0.f;
      for (int sl = 0; sl < p.kb; sl++) v += s_red[(tl * p.kb + sl) * 16 * B + rb];
      s_val[idx] = v;
    }
    __syncthreads();
  }
  ckpt(kc, 4);
  v2_epilogue(a, B, p.t0, p.nt, s_val, B, kc);
  ckpt(kc, 5);
}

// int8 weights on the s8 MMA with the four-part activation (as gemv2_s8_t).
template <int NCH>
__device__ __noinline__ void gemv_cl_s8_t(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  constexpr int PC = cl_pc<FMT_INT8>();
  const V2Plan p = kc.pring[kc.seq % NDESC];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
  float *s_scl = reinterpret_cast<float *>(smem + SM_R_OFF);
  float *s_red = s_scl + 64;   // [nt * ks][16][B]
  uint32_t *s_xw = reinterpret_cast<uint32_t *>(smem + SM_X_OFF);
  const uint2 *s_xf = reinterpret_cast<const uint2 *>(s_xw);
  const int np = cl_npieces(p, warp);

  ckpt(kc, 11);
  if (lane == 0) cl_start<FMT_INT8>(a, p, warp, np, kc, smem);
  __syncwarp();
  ckpt(kc, 0);
  if (p.nt == 0) return;
  {
    const int mq = (B * (a.K >> 2) + NTHREADS - 1) / NTHREADS;
    if (mq <= 1) stage_x_s8<1>(a, B, NCH, 0, a.K, s_scl, s_xw, s_red, 0, kc);
    else if (mq <= 2) stage_x_s8<2>(a, B, NCH, 0, a.K, s_scl, s_xw, s_red, 0, kc);
    else if (mq <= 4) stage_x_s8<4>(a, B, NCH, 0, a.K, s_scl, s_xw, s_red, 0, kc);
    else stage_x_s8<8>(a, B, NCH, 0, a.K, s_scl, s_xw, s_red, 0, kc);
  }
  __syncthreads();
  ckpt(kc, 2);

  // column pair (2 tig, 2 tig + 1) of chunk j = parts (2 (tig & 1), +1) of
  // batch row 2 j + tig / 2
  const float wlo = (tig & 1) ? (1.0f / 16384.0f) : 1.0f, whi = (tig & 1) ? (1.0f / 2097152.0f) : (1.0f / 128.0f);
  int acc[4][NCH][4];
#pragma unroll
  for (int u = 0; u < 4; u++)
#pragma unroll
    for (int j = 0; j < NCH; j++) acc[u][j][0] = acc[u][j][1] = acc[u][j][2] = acc[u][j][3] = 0;
  for (int q = 0; q < np; q++) {
    const ClPiece pc = cl_piece(p, PC, warp, q);
    const char *slot = cl_wait(kc, smem, warp, q);
    if (q == 0) ckpt(kc, 12);
    int i = 0;
    for (; i + 4 <= pc.n; i += 4) {
      uint4 wv[4];
#pragma unroll
      for (int u = 0; u < 4; u++) wv[u] = *reinterpret_cast<const uint4 *>(slot + (i + u) * 512 + lane * 16);
#pragma unroll
      for (int u = 0; u < 4; u++)
#pragma unroll
        for (int j = 0; j < NCH; j++) {
          const uint2 bx = s_xf[((pc.c0 + i + u) * NCH + j) * 32 + lane];
          mma_s8(acc[u][j], wv[u], bx.x, bx.y);
        }
    }
    for (; i < pc.n; i++) {
      const uint4 wv = *reinterpret_cast<const uint4 *>(slot + i * 512 + lane * 16);
#pragma unroll
      for (int j = 0; j < NCH; j++) {
        const uint2 bx = s_xf[((pc.c0 + i) * NCH + j) * 32 + lane];
        mma_s8(acc[0][j], wv, bx.x, bx.y);
      }
    }
    cl_release<FMT_INT8>(a, p, warp, q, np, kc, smem);
    if (pc.c0 + pc.n == (pc.s + 1) * p.kc) {   // the unit's last piece: its 16 rows out
      const int un = pc.tl * p.kb + pc.s;
#pragma unroll
      for (int j = 0; j < NCH; j++) {
        const int i0 = acc[0][j][0] + acc[1][j][0] + acc[2][j][0] + acc[3][j][0];
        const int i1 = acc[0][j][1] + acc[1][j][1] + acc[2][j][1] + acc[3][j][1];
        const int i2 = acc[0][j][2] + acc[1][j][2] + acc[2][j][2] + acc[3][j][2];
        const int i3 = acc[0][j][3] + acc[1][j][3] + acc[2][j][3] + acc[3][j][3];
        float r0 = (float)i0 * wlo + (float)i1 * whi;   // row gid
        float r1 = (float)i2 * wlo + (float)i3 * whi;   // row gid + 8
        r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
        r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
        const int b = 2 * j + (tig >> 1);
        if ((tig & 1) == 0 && b < B) {
          const float sx = s_scl[4 + b];
          s_red[(un * 16 + gid) * B + b] = r0 * sx;
          s_red[(un * 16 + gid + 8) * B + b] = r1 * sx;
        }
#pragma unroll
        for (int u = 0; u < 4; u++) acc[u][j][0] = acc[u][j][1] = acc[u][j][2] = acc[u][j][3] = 0;
      }
    }
  }
  ckpt_w(kc, 24);
  if (lane == 0) cl_issue_ahead(kc, smem, warp);
  __syncthreads();
  ckpt(kc, 3);
  float *s_val = s_red;
  if (p.kb > 1) {   // a tile's slices, in slice order
    s_val = s_red + p.nt * p.kb * 16 * B;
    for (int idx = tid; idx < p.nt * 16 * B; idx += NTHREADS) {
      const int rb = idx % (16 * B), tl = idx / (16 * B);
      float v = 0.f;
      for (int sl = 0; sl < p.kb; sl++) v += s_red[(tl * p.kb + sl) * 16 * B + rb];
      s_val[idx] = v;
    }
    __syncthreads();
  }
  ckpt(kc, 4);
  v2_epilogue(a, B, p.t0, p.nt, s_val, B, kc);
  ckpt(kc, 5);
}

template <int FMT>
QTB_DEV void gemv_cl_f(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  if (FMT == FMT_INT8 && a.parts == 4) {
    switch (a.nch) {
      case 1: gemv_cl_s8_t<1>(a, B, smem, kc); return;
      case 2: gemv_cl_s8_t<2>(a, B, smem, kc); return;
    }
  } else if (FMT == FMT_BF16 && a.parts == 4) {
    switch (a.nch) {
      case 1: gemv_cl_t<FMT, 1, 4>(a, B, smem, kc); return;
      case 2: gemv_cl_t<FMT, 2, 4>(a, B, smem, kc); return;
    }
  } else if (a.parts == 2 && FMT != FMT_BF16 && FMT != FMT_INT8) {
    switch (a.nch) {
      case 1: gemv_cl_t<FMT, 1, 2>(a, B, smem, kc); return;
    }
  }
  if (threadIdx.x == 0) raise_err(kc, ERR_BAD_STAGE, 5000 + a.nch * 16 + a.parts);
}

// ============================================ GEMV stage on tcgen05 =======
//
// Large batches (5..64 rows) with bf16 or int8 weights, in two phases.
//  1. Prep: CTA b (b < B) turns activation row b into rows of the B operand in
//     a global staging buffer `xop` (K-major, 128-byte swizzle, one block of
//     N x 128 bytes per 128-byte K chunk), with the RMSNorm gain applied: int8
//     weights take four signed 8-bit parts per value, x g = sx (a0 + a1 2^-7 +
//     a2 2^-14 + a3 2^-21) with sx = max|x g| / 127 over the row (operand row
//     4 b + p, kind::i8, exact s32 sums); bf16 weights take bf16 hi + lo parts
//     (operand row 2 b + p, kind::f16, f32 sums).  It stores sx and the row's
//     1/rms (1 without a norm) in xsc[b], xsc[64 + b], then counts itself on
//     ctl->ibar.  Every other CTA meanwhile bulk-copies its first weight
//     chunks.  The row goes through shared memory in rolled loops: the phase
//     runs once per stage, and straight-line code that runs once is fetched
//     into a cold instruction cache line by line.
//  2. Stream: once B rows are counted, a CTA owns a run of 128-row tiles (its
//     row group) over one k-slice (host plan V2Plan: t0, nt, kb / kc = first
//     128-byte chunk and chunk count, pair = slice).  Thread 0 bulk-copies each
//     chunk's pre-swizzled weight tile (128 rows x 128 bytes, 16 KB) and the
//     matching operand block (N x 128 bytes) into one of TC_NSLOT slots and
//     issues four MMAs (M 128, N = parts x padded batch, 32 bytes of K each)
//     into the TMEM accumulator; a slot is refilled once the MMAs reading it
//     have completed (tcgen05.commit -> mbarrier).  All warps read the
//     accumulator back (warp w: TMEM lanes 32 (w % 4) .., batch half w / 4).
//  3. With one slice the epilogue runs at once; with several, partial sums go
//     to ws and the slices of a tile add them in slice order (deterministic)
//     and run it.
QTB_HOST_DEV constexpr int tc_parts(int fmt) { return fmt == FMT_INT8 ? 4 : 2; }
QTB_HOST_DEV constexpr int tc_kchunk(int fmt) { return fmt == FMT_INT8 ? 128 : 64; }   // K per 128-byte chunk
// Batch rows padded to a multiple of 8 (N = parts x rows a multiple of 16,
// each warp's half of the batch a whole number of float4s).
QTB_HOST_DEV constexpr int tc_bpad(int fmt, int B) { return (void)fmt, (B + 7) & ~7; }
// Bytes of the operand staging buffer for K columns (B <= 64).
QTB_HOST_DEV constexpr size_t tc_xop_bytes(int fmt, int K) {
  return (size_t)(K / tc_kchunk(fmt)) * tc_parts(fmt) * 64 * 128;
}

QTB_HOST_DEV uint32_t tc_sw128(int n, int kb) {   // byte offset of (row n, byte kb of a 128-byte K chunk)
  return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((((kb >> 4) ^ (n & 7)) << 4) | (kb & 15)));
}

QTB_DEV void cp_async16(void *dst_smem, const void *src_gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src_gmem) : "memory");
}
QTB_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Phase 1 for row b (the whole CTA): see the comment above.  `row` is K floats
// of shared memory, s_red 16 floats.
template <int FMT>
__device__ __noinline__ void tc_prep_row(const GemvArgs &a, int b, int N, float *row, float *s_red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nq = a.K >> 2;
  const float *src = a.x + (size_t)b * a.ldx;
#pragma unroll 1
  for (int q = tid; q < nq; q += NTHREADS) cp_async16(row + 4 * q, src + 4 * q);
  cp_async_wait_all();
  __syncthreads();
  float ss = 0.f, m = 0.f;
#pragma unroll 1
  for (int q = tid; q < nq; q += NTHREADS) {
    const float4 v = *reinterpret_cast<const float4 *>(row + 4 * q);
    const float4 g = a.norm_w ? __ldg(reinterpret_cast<const float4 *>(a.norm_w) + q) : make_float4(1.f, 1.f, 1.f, 1.f);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x * g.x), fabsf(v.y * g.y)), fmaxf(fabsf(v.z * g.z), fabsf(v.w * g.w))));
  }
  ss = warp_sum(ss);
  m = warp_max(m);
  if (lane == 0) { s_red[warp] = ss; s_red[NWARPS + warp] = m; }
  __syncthreads();
  float tot = 0.f, mx = 0.f;
#pragma unroll
  for (int w = 0; w < NWARPS; w++) { tot += s_red[w]; mx = fmaxf(mx, s_red[NWARPS + w]); }
  const float sx = fmaxf(mx, 1e-30f) * (1.0f / 127.0f), rs = __frcp_rn(sx);
  if (tid == 0) {
    a.xsc[b] = sx;
    a.xsc[64 + b] = a.norm_w ? 1.0f / sqrtf(tot / (float)a.K + a.eps) : 1.0f;
  }
  uint8_t *xop = a.xop;
#pragma unroll 1
  for (int q = tid; q < nq; q += NTHREADS) {
    const float4 v = *reinterpret_cast<const float4 *>(row + 4 * q);
    const float4 g = a.norm_w ? __ldg(reinterpret_cast<const float4 *>(a.norm_w) + q) : make_float4(1.f, 1.f, 1.f, 1.f);
    const float e[4] = {v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w};
    if (FMT == FMT_INT8) {
      uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float r = fminf(fmaxf(e[k] * rs, -127.f), 127.f);
        // fixed point r 2^21 as a leading part and three balanced base-128 digits
        int I = __float2int_rn(r * 2097152.f);
        const int d3 = ((I + 64) & 127) - 64;
        I = (I - d3) >> 7;
        const int d2 = ((I + 64) & 127) - 64;
        I = (I - d2) >> 7;
        const int d1 = ((I + 64) & 127) - 64;
        const int a0 = (I - d1) >> 7;
        w[0] |= ((uint32_t)a0 & 0xffu) << (8 * k);
        w[1] |= ((uint32_t)d1 & 0xffu) << (8 * k);
        w[2] |= ((uint32_t)d2 & 0xffu) << (8 * k);
        w[3] |= ((uint32_t)d3 & 0xffu) << (8 * k);
      }
      const int k0 = 4 * q, c = k0 >> 7, kb = k0 & 127;
#pragma unroll
      for (int p = 0; p < 4; p++)
        __stcg(reinterpret_cast<unsigned *>(xop + (size_t)c * N * 128 + tc_sw128(4 * b + p, kb)), w[p]);
    } else {
      uint32_t hi[2], lo[2];
#pragma unroll
      for (int k = 0; k < 2; k++) {
        const uint32_t h0 = f32_to_bf16_rn(e[2 * k]), h1 = f32_to_bf16_rn(e[2 * k + 1]);
        const uint32_t l0 = f32_to_bf16_rn(e[2 * k] - __uint_as_float(h0 << 16));
        const uint32_t l1 = f32_to_bf16_rn(e[2 * k + 1] - __uint_as_float(h1 << 16));
        hi[k] = h0 | (h1 << 16);
        lo[k] = l0 | (l1 << 16);
      }
      const int kbyte = 8 * q, c = kbyte >> 7, kb = kbyte & 127;
      __stcg(reinterpret_cast<uint2 *>(xop + (size_t)c * N * 128 + tc_sw128(2 * b, kb)), make_uint2(hi[0], hi[1]));
      __stcg(reinterpret_cast<uint2 *>(xop + (size_t)c * N * 128 + tc_sw128(2 * b + 1, kb)), make_uint2(lo[0], lo[1]));
    }
  }
  // the operand is read by other CTAs' bulk copies (async proxy)
  fence_proxy_async();
}

// Final value of (row, batch b): 1/rms, row scale, bias, then the epilogue
// (warp-uniform in b: SWIGLU exchanges the interleaved gate / up rows, which
// sit in neighbouring lanes).
QTB_DEV void tc_out(const GemvArgs &a, int B, int b, int row, float v, float inv) {
  v *= inv;
  if (a.row_scale) v *= __ldg(a.row_scale + row);
  if (a.bias) v += __ldg(a.bias + row);
  if (a.epi == EPI_SWIGLU) {
    const float up = __shfl_xor_sync(0xffffffffu, v, 1);
    if ((row & 1) == 0 && b < B) __stcg(a.y + (size_t)b * a.ldy + (row >> 1), __fdividef(v, 1.0f + expf(-v)) * up);
  } else if (b < B) {
    float *yp = a.y + (size_t)b * a.ldy + row;
    if (a.epi == EPI_RESID) __stcg(yp, __ldcg(yp) + v);
    else __stcg(yp, v);
  }
}

template <int FMT>
__device__ __noinline__ void gemv_tc_t(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  const V2Plan pl = kc.pring[kc.seq % NDESC];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = tc_parts(FMT), Bp = tc_bpad(FMT, B), N = P * Bp, Bh = Bp / 2;
  const int S = a.S, s = pl.pair, t0 = pl.t0, nt = pl.nt, kcn = pl.kc;
  const int NKC = a.K / tc_kchunk(FMT);
  const int L = nt * kcn;
  const uint32_t XB = (uint32_t)N * 128u;   // operand bytes per chunk
  // slot regions from the first 1024-byte aligned byte of dynamic smem
  const uint32_t base_u = smem_u32(smem);
  char *tcb = smem + ((1024u - (base_u & 1023u)) & 1023u);
  char *wring = tcb;
  char *xring = tcb + TC_XR_OFF;
  float *s_sx = reinterpret_cast<float *>(smem + TC_SCR_OFF);   // [64]
  float *s_red = s_sx + 64;                                     // [64]
  float *s_inv = s_red + 64;                                    // [64]
  int *s_flag = reinterpret_cast<int *>(s_inv + 64);            // [4]
  unsigned long long *s_key = reinterpret_cast<unsigned long long *>(s_flag + 4);   // [4][64]
  const uint64_t pol = a.evict_last ? kc.pol_last : kc.pol_first;
  const unsigned F0 = kc.tc_issued;   // fills of earlier tcgen05 stages (all consumed)
  const unsigned g0 = kc.tc_waited;   // accumulator uses so far (buffer g & 1 for the g-th)
  const unsigned ib_target = kc.ibar_target + (unsigned)B;

  // thread 0: fill f (tile t0 + f / kcn, chunk kb + f % kcn) into slot
  // (F0 + f) % TC_NSLOT once the MMAs that last read the slot are done: the
  // weight tile now, the operand block now or (first fills) after the prep
  auto issue_w = [&](int f) -> bool {
    const unsigned F = F0 + (unsigned)f, slot = F % TC_NSLOT, use = F / TC_NSLOT;
    if (use > 0 && !mbar_wait(kc.tcempty + slot, (use - 1) & 1u, WAIT_LIMIT_CYCLES)) {
      raise_err(kc, ERR_MBAR_TIMEOUT, 2000 + f);
      return false;
    }
    const int tile = t0 + f / kcn, chunk = pl.kb + f % kcn;
    mbar_arrive_expect_tx(kc.tcfull + slot, TC_SLOT_BYTES + XB);
    bulk_g2s_hint(wring + slot * TC_SLOT_BYTES, a.wtc + ((size_t)tile * NKC + chunk) * TC_SLOT_BYTES, TC_SLOT_BYTES,
                  kc.tcfull + slot, pol);
    kc.tc_issued = F + 1u;
    return true;
  };
  auto issue_x = [&](int f) {
    const unsigned slot = (F0 + (unsigned)f) % TC_NSLOT;
    const int chunk = pl.kb + f % kcn;
    bulk_g2s(xring + slot * TC_XSLOT_BYTES, a.xop + (size_t)chunk * XB, XB, kc.tcfull + slot);
  };
  // the next tcgen05 stage's weight tiles (this CTA's share) into L2 while
  // this one runs: its first copies then come from L2 instead of HBM.  Looks
  // two stages ahead, at descriptors that have landed only.
  if (tid == 64) {
    for (unsigned k = 1; k <= 2; k++) {
      const unsigned nx = kc.seq + k;
      if (nx >= kc.n_total) break;
      const int sl = (int)(nx % NDESC);
      if (!mbar_test(kc.dbars + sl, (nx / NDESC) & 1u)) break;
      const Stage &ns = kc.dring[sl];
      if (ns.kind != ST_GEMV) continue;
      if (ns.g.tc) {
        const V2Plan &np = kc.pring[sl];
        const int nkc = ns.g.K / tc_kchunk(ns.g.fmt);
        for (int ti = 0; ti < np.nt; ti++)
          prefetch_l2(ns.g.wtc + ((size_t)(np.t0 + ti) * nkc + np.kb) * TC_SLOT_BYTES, (uint32_t)np.kc * TC_SLOT_BYTES);
      }
      break;
    }
  }
  const int nfirst = min(TC_NSLOT, L);
  if (tid == 0 && nt > 0) {
    fence_proxy_async_smem();   // the slots were last written through the generic proxy (other stages)
    for (int f = 0; f < nfirst; f++)
      if (!issue_w(f)) break;
  }
  ckpt(kc, 0);
  // ---- phase 1: this CTA's activation row (the row buffer is the operand
  // slot region, idle until the operand copies below) ----
  if ((int)blockIdx.x < B) {
    tc_prep_row<FMT>(a, blockIdx.x, N, reinterpret_cast<float *>(xring), s_red);
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      atom_add_release_gpu(&kc.ctl->ibar, 1u);
    }
  }
  ckpt(kc, 1);
  // ---- the B rows are in place (bounded wait; warp 1 polls, so thread 0's
  // weight copies in flight do not hold the poll back) ----
  if (tid == 32) {
    const long long w0 = clock64();
    while ((int)(ld_acquire_gpu(&kc.ctl->ibar) - ib_target) < 0) {
      if (clock64() - w0 > WAIT_LIMIT_CYCLES || ld_acquire_gpu((const unsigned *)&kc.ctl->err)) {
        raise_err(kc, ERR_BARRIER_TIMEOUT, 6000 + (int)blockIdx.x);
        break;
      }
    }
  }
  __syncthreads();
  if (tid == 0) kc.ibar_target = ib_target;
  if (kc.local_err) {
    // the CTA leaves together; the first fills' operand copies still go out
    // so that every fill issued completes (the stale operand is never used)
    if (tid == 0 && nt > 0)
      for (int f = 0; f < nfirst && F0 + (unsigned)f < kc.tc_issued; f++) issue_x(f);
    return;
  }
  ckpt(kc, 2);
  if (nt == 0) return;
  if (tid < Bp) {
    s_sx[tid] = (tid < B) ? __ldcg(a.xsc + tid) : 0.f;
    s_inv[tid] = (tid < B) ? __ldcg(a.xsc + 64 + tid) : 0.f;
  }
  if (tid == 0) {
    fence_proxy_async();        // the operand, written by other CTAs, is read by bulk copies
    fence_proxy_async_smem();   // the row buffer was written through the generic proxy
    for (int f = 0; f < nfirst; f++) issue_x(f);
  }

  const uint32_t idesc = (FMT == FMT_INT8) ? umma_idesc(2u, 1u, (uint32_t)N) : umma_idesc(1u, 1u, (uint32_t)N);
  const uint32_t wr_u = smem_u32(wring), xr_u = smem_u32(xring);
  // thread 0: the MMAs of tile i into accumulator buffer (g0 + i) & 1
  auto mma_tile = [&](int i) {
    const unsigned g = g0 + (unsigned)i;
    const uint32_t d = kc.tmem + (g & 1u) * (uint32_t)TC_ACC_COLS;
    for (int c = 0; c < kcn; c++) {
      const int f = i * kcn + c;
      const unsigned F = F0 + (unsigned)f, slot = F % TC_NSLOT;
      if (!mbar_wait(kc.tcfull + slot, (F / TC_NSLOT) & 1u, WAIT_LIMIT_CYCLES)) {
        raise_err(kc, ERR_MBAR_TIMEOUT, 3000 + f);
        break;
      }
      kc.tc_done = F + 1u;
      tc_fence_after();
      const uint32_t ab = wr_u + slot * TC_SLOT_BYTES, bb = xr_u + slot * TC_XSLOT_BYTES;
#pragma unroll
      for (int ks = 0; ks < 4; ks++) {
        const uint64_t ad = umma_desc_sw128(ab + 32u * ks), bd = umma_desc_sw128(bb + 32u * ks);
        if (FMT == FMT_INT8) umma_i8(d, ad, bd, idesc, (c | ks) != 0);
        else umma_bf16(d, ad, bd, idesc, (c | ks) != 0);
      }
      umma_commit(kc.tcempty + slot);
      if (f + TC_NSLOT < L) {   // refill this slot
        if (!issue_w(f + TC_NSLOT)) break;
        issue_x(f + TC_NSLOT);
      }
    }
    umma_commit(kc.tcacc + (g & 1u));
    kc.tc_committed = g + 1u;
  };
  __syncthreads();   // s_sx, s_inv
  if (tid == 0 && !kc.local_err) mma_tile(0);

  const int q4 = warp & 3, hh = warp >> 2;
  const int rl = 32 * q4 + lane;   // this thread's row within the tile
  const float c7 = 1.0f / 128.0f, c14 = 1.0f / 16384.0f, c21 = 1.0f / 2097152.0f;
  for (int i = 0; i < nt; i++) {
    const int t = t0 + i;
    const unsigned g = g0 + (unsigned)i;
    // the next tile's MMAs go into the other buffer while this one is read
    if (tid == 0 && i + 1 < nt && !kc.local_err) mma_tile(i + 1);
    ckpt(kc, 12);
    if (i < 3) ckpt(kc, 17 + 4 * i);
    const bool landed = mbar_wait(kc.tcacc + (g & 1u), (g >> 1) & 1u, WAIT_LIMIT_CYCLES);
    if (!landed && lane == 0) raise_err(kc, ERR_MBAR_TIMEOUT, 4000 + i);
    tc_fence_after();
    ckpt(kc, 13);
    if (i < 3) ckpt(kc, 18 + 4 * i);
    // batch rows [hh * Bh, hh * Bh + Bh) of row rl, PER per 32-column TMEM
    // load: a rolled loop over the loads, each load's values unrolled (this
    // code runs once per stage, and code that runs once is fetched line by
    // line into a cold instruction cache)
    constexpr int PER = (FMT == FMT_INT8) ? 8 : 16;
    const int row = 128 * t + rl;
    const float rsc = (S == 1 && a.row_scale) ? __ldg(a.row_scale + row) : 1.f;
    const float bia = (S == 1 && a.bias) ? __ldg(a.bias + row) : 0.f;
#pragma unroll 1
    for (int j = 0; j < 32 / PER; j++) {
      if (PER * j >= Bh) break;
      const int bb0 = hh * Bh + PER * j;
      uint32_t r[32];
      tmem_ld32(kc.tmem + (g & 1u) * (uint32_t)TC_ACC_COLS + ((uint32_t)(32 * q4) << 16) + (uint32_t)(P * bb0), r);
      float v[PER];
#pragma unroll
      for (int u = 0; u < PER; u++) {
        if (FMT == FMT_INT8) {
          v[u] = (((float)(int)r[4 * u + 3] * c21 + (float)(int)r[4 * u + 2] * c14) + (float)(int)r[4 * u + 1] * c7) +
                 (float)(int)r[4 * u];
          const int b = bb0 + u;
          v[u] *= (b < B) ? s_sx[b] : 0.f;
        } else {
          v[u] = __uint_as_float(r[2 * u]) + __uint_as_float(r[2 * u + 1]);
        }
      }
      const int nu = min(PER, Bh - PER * j);   // this half's rows in the load (a multiple of 4)
      if (S > 1) {
        // this slice's partial sums of the tile; added up after the last tile
        float *wsp = a.ws + (((size_t)t * S + s) * 128 + rl) * Bp + bb0;
#pragma unroll
        for (int u = 0; u < PER; u += 4)
          if (u < nu) __stcg(reinterpret_cast<float4 *>(wsp + u), make_float4(v[u], v[u + 1], v[u + 2], v[u + 3]));
      } else if (a.epi == EPI_ARGMAX) {
        // per batch row: this warp's 32 rows now, the four lane quarters below
#pragma unroll 1
        for (int u = 0; u < nu; u++) {
          const int b = bb0 + u;
          unsigned long long k = 0ull;
          if (b < B) {
            float x = v[u] * s_inv[b] * rsc + bia;
            if (a.gen) x = codec_logit(a.gen, b, row, x);
            k = amax_key(x, row);
          }
#pragma unroll
          for (int m = 16; m > 0; m >>= 1) {
            const unsigned long long o = shfl_xor_u64(k, m);
            k = o > k ? o : k;
          }
          if (lane == 0) s_key[q4 * 64 + b] = k;
        }
      } else if (a.epi == EPI_SWIGLU) {
        float *yh = a.y + (row >> 1);
#pragma unroll
        for (int u = 0; u < PER; u++) {
          if (u >= nu) break;
          const int b = bb0 + u;
          const float x = (v[u] * s_inv[b]) * rsc + bia;
          const float up = __shfl_xor_sync(0xffffffffu, x, 1);
          if ((row & 1) == 0 && b < B) __stcg(yh + (size_t)b * a.ldy, __fdividef(x, 1.0f + expf(-x)) * up);
        }
      } else if (a.epi == EPI_RESID) {
#pragma unroll
        for (int u = 0; u < PER; u++) {
          const int b = bb0 + u;
          if (u < nu && b < B) {
            float *yp = a.y + (size_t)b * a.ldy + row;
            __stcg(yp, __ldcg(yp) + ((v[u] * s_inv[b]) * rsc + bia));
          }
        }
      } else {
#pragma unroll
        for (int u = 0; u < PER; u++) {
          const int b = bb0 + u;
          if (u < nu && b < B) __stcg(a.y + (size_t)b * a.ldy + row, (v[u] * s_inv[b]) * rsc + bia);
        }
      }
    }
    tc_fence_before();
    if (i < 3) ckpt(kc, 19 + 4 * i);
    if (S == 1 && a.epi == EPI_ARGMAX) {
      __syncthreads();
      for (int idx = tid; idx < 8 * B; idx += NTHREADS) {
        const int b = idx % B, sub = idx / B;
        unsigned long long best = 0ull;
        if (sub == 0)
          for (int qq = 0; qq < 4; qq++) best = s_key[qq * 64 + b] > best ? s_key[qq * 64 + b] : best;
        a.amax_ws[(size_t)(8 * t + sub) * B + b] = best;
      }
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        s_flag[1] = (atomicAdd(a.amax_sem, 8u) + 8u == (unsigned)(a.rows >> 4));
      }
      __syncthreads();
      if (s_flag[1]) argmax_finish(a, B, kc);
    }
    // this buffer may take tile i + 2
    if (__syncthreads_or(kc.local_err)) return;   // copies and MMAs in flight are drained on the way out
    if (tid == 0) kc.tc_waited = g + 1u;
    ckpt(kc, 14);
    if (i < 3) ckpt(kc, 20 + 4 * i);
  }
  if (tid == 0) kc.tc_issued = F0 + (unsigned)L;
  if (S == 1) return;

  // ---- split K: every slice CTA of a tile adds up its share of 16-row
  // sub-tiles (st = s, s + S, ...) over the slices, in slice order ----
  __threadfence();
  __syncthreads();   // partial sums and sums of squares stored
  if (tid == 0)
    for (int i = 0; i < nt; i++) atom_add_release_gpu(a.sem + a.sem_off + t0 + i, 1u);
  if (s >= 8) return;   // no sub-tile left for this slice
  // each program iteration adds S to the counters (zeroed at launch): wait
  // for every slice of this CTA's tiles
  const unsigned target = (unsigned)S * (kc.seq / (unsigned)kc.n_stages + 1u);
  if (tid == 0) {
    const long long w0 = clock64();
    for (int i = 0; i < nt && !kc.local_err; i++) {
      const unsigned *tsem = a.sem + a.sem_off + t0 + i;
      while ((int)(ld_acquire_gpu(tsem) - target) < 0) {
        if (clock64() - w0 > WAIT_LIMIT_CYCLES || ld_acquire_gpu((const unsigned *)&kc.ctl->err)) {
          raise_err(kc, ERR_BARRIER_TIMEOUT, 5000 + t0 + i);
          break;
        }
      }
    }
  }
  ckpt(kc, 16);
  if (__syncthreads_or(kc.local_err)) return;
  __threadfence();
  // work items (tile i, sub-tile st of this slice): thread = row r of the
  // sub-tile x batch rows 4 bq .. 4 bq + 3
  const int per_tile = (8 - s + S - 1) / S;   // sub-tiles s, s + S, ... < 8
  const int nitems = nt * per_tile;
  const int r = tid & 15, bq = tid >> 4;
  const bool act = 4 * bq < Bp;
  const size_t sstride = (size_t)128 * Bp;
  for (int w = 0; w < nitems; w++) {
    const int i = w / per_tile, st = s + S * (w - i * per_tile);
    const int t = t0 + i;
    const int rrow = 128 * t + 16 * st + r;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (act) {
      const float *src = a.ws + (((size_t)t * S) * 128 + 16 * st + r) * Bp + 4 * bq;
      int s2 = 0;
      for (; s2 + 8 <= S; s2 += 8) {   // eight slices' loads in flight, added in slice order
        float4 p[8];
#pragma unroll
        for (int k = 0; k < 8; k++) p[k] = ld_cg4(src + (s2 + k) * sstride);
#pragma unroll
        for (int k = 0; k < 8; k++) { acc.x += p[k].x; acc.y += p[k].y; acc.z += p[k].z; acc.w += p[k].w; }
      }
      for (; s2 < S; s2++) {
        const float4 p0 = ld_cg4(src + s2 * sstride);
        acc.x += p0.x; acc.y += p0.y; acc.z += p0.z; acc.w += p0.w;
      }
    }
    const float vv[4] = {acc.x, acc.y, acc.z, acc.w};
    if (a.epi == EPI_ARGMAX) {
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int b = 4 * bq + k;
        unsigned long long key = 0ull;
        if (act && b < B) {
          float v = vv[k] * s_inv[b] * (a.row_scale ? __ldg(a.row_scale + rrow) : 1.f) + (a.bias ? __ldg(a.bias + rrow) : 0.f);
          if (a.gen) v = codec_logit(a.gen, b, rrow, v);
          key = amax_key(v, rrow);
        }
#pragma unroll
        for (int m = 8; m > 0; m >>= 1) {
          const unsigned long long o = shfl_xor_u64(key, m);
          key = o > key ? o : key;
        }
        if (r == 0 && act && b < B) a.amax_ws[(size_t)(8 * t + st) * B + b] = key;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int b = 4 * bq + k;
        // (SWIGLU pairs rows r, r ^ 1: neighbouring lanes of one 16-lane group)
        tc_out(a, act ? B : 0, b, rrow, vv[k], (act && b < Bp) ? s_inv[b] : 0.f);
      }
    }
  }
  const int nsub = nitems;
  if (a.epi == EPI_ARGMAX) {
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      s_flag[1] = (atomicAdd(a.amax_sem, (unsigned)nsub) + (unsigned)nsub == (unsigned)(a.rows >> 4));
    }
    __syncthreads();
    if (s_flag[1]) argmax_finish(a, B, kc);
  }
  ckpt(kc, 15);
}

template <int FMT>
QTB_DEV void gemv2_stage_f(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  if (FMT == FMT_INT8 && a.parts == 4) {
    switch (a.nch) {
      case 1: gemv2_s8_t<1>(a, B, smem, kc); return;
      case 2: gemv2_s8_t<2>(a, B, smem, kc); return;
    }
  } else if (FMT == FMT_BF16 && a.parts == 4) {
    switch (a.nch) {
      case 1: gemv2_stage_t<FMT, 1, 4>(a, B, smem, kc); return;
      case 2: gemv2_stage_t<FMT, 2, 4>(a, B, smem, kc); return;
    }
  } else if (a.parts == 2 && FMT != FMT_BF16 && FMT != FMT_INT8) {
    switch (a.nch) {
      case 1: gemv2_stage_t<FMT, 1, 2>(a, B, smem, kc); return;
    }
  }
  if (threadIdx.x == 0) raise_err(kc, ERR_BAD_STAGE, 1000 + a.nch * 16 + a.parts);
}

template <int FMT>
QTB_DEV void gemv_stage_f(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  if (a.cl) { gemv_cl_f<FMT>(a, B, smem, kc); return; }
  if (a.v2) { gemv2_stage_f<FMT>(a, B, smem, kc); return; }
  if (FMT == FMT_BF16 || FMT == FMT_INT8) {
    // large batches of bf16 / int8 weights always run on tcgen05
    if (a.tc) gemv_tc_t<FMT>(a, B, smem, kc);
    else if (threadIdx.x == 0) raise_err(kc, ERR_BAD_STAGE, 2000 + FMT);
    return;
  }
  // large batches of 4-bit weights: the k-sliced mma.sync path
  if (a.parts == 2) {
    switch (a.nch) {
      case 1: if (FMT != FMT_BF16) { gemv_stage_t<FMT, 1, 2>(a, B, smem, kc); return; } break;
      case 2: if (FMT != FMT_BF16) { gemv_stage_t<FMT, 2, 2>(a, B, smem, kc); return; } break;
      case 4: if (FMT != FMT_BF16) { gemv_stage_t<FMT, 4, 2>(a, B, smem, kc); return; } break;
      case 8: gemv_stage_t<FMT, 8, 2>(a, B, smem, kc); return;
      case 16: gemv_stage_t<FMT, 16, 2>(a, B, smem, kc); return;
    }
  }
  if (threadIdx.x == 0) raise_err(kc, ERR_BAD_STAGE, a.nch * 16 + a.parts);
}

QTB_DEV void gemv_stage(const GemvArgs &a, int B, char *smem, KCtx &kc) {
  switch (a.fmt) {
    case FMT_BF16: gemv_stage_f<FMT_BF16>(a, B, smem, kc); break;
    case FMT_INT8: gemv_stage_f<FMT_INT8>(a, B, smem, kc); break;
    case FMT_Q4_0: gemv_stage_f<FMT_Q4_0>(a, B, smem, kc); break;
    case FMT_INT4G: gemv_stage_f<FMT_INT4G>(a, B, smem, kc); break;
    default: if (threadIdx.x == 0) raise_err(kc, ERR_BAD_STAGE, a.fmt); break;
  }
}

// =========================================================== ATTN stage ====
//
// Work item = (slot b, kv head g, split sp).  Every CTA of an item recomputes
// the normed + roped query heads 2g, 2g+1 (qwen_rms_norm_per_head,
// qwen_tts_kernels.c:486-577; apply_rope_neox_inplace, qwen_tts_talker.c:
// 203-251) and the new K/V of head g; the CTA whose split holds the newest
// page also appends K/V (bf16 by truncation, qwen_tts_talker.c:612-615) into
// the slot's page with 16-byte stores.  Pages are staged into shared memory
// by 1D bulk copies (cp.async.bulk, mbarrier completion) through a ring of 4
// buffers, or 16 in programs whose weight ring is idle (large batches).  The
// CTA's 8 warps work as 4 pairs (the two query heads of the GQA group), pair
// p on pages p, p + 4, ..., each warp with its own online softmax, merged in
// warp order at the end.  Scores use the reference's order (dot, then *
// scale); the softmax is the online recurrence of qwen_causal_attention_bf16kv
// (qwen_tts_kernels.c:3704-3846) applied per page.  When an item has several
// splits the last finishing CTA combines them (deterministic order).
// Items go to CTAs either statically (item = CTA + k * grid: at most one per
// CTA in small batches) or, for large batches, from a grid-wide counter in the
// dense order of attn_prefix, so CTAs that drew short sequences take more.
// Either way an item's arithmetic does not depend on the CTA: results are
// identical run to run.

// The bf16 rows of the new token come first: they are read as 16-byte
// vectors for the page store, so they must sit on 16-byte boundaries.
struct __align__(16) AttnSmem {
  uint16_t knew[HD];
  uint16_t vnew[HD];
  float q[2][HD];
  int pre[65];                   // dynamic order: first item of each batch slot, items in all at [B]
  int next;                      // dynamic order: the CTA's next item
  int flag;
};
static_assert(sizeof(AttnSmem) <= 2048, "attention scratch overlaps the page buffers");
// per-warp softmax states for the end-of-split combine: [NWARPS][HD] + [NWARPS][2]
constexpr int ATT_COMB_OFF = 2048 + ATT_NBUF * ATT_PAGE_BYTES;
static_assert(ATT_COMB_OFF + NWARPS * (HD + 2) * 4 <= SM_X2_BYTES, "page ring exceeds the attention region");
static_assert(NWARPS == 2 * ATT_NBUF, "one warp pair (the two heads of a GQA group) per page buffer group");
static_assert((ATT_NBUF_MAX - ATT_NBUF) * ATT_PAGE_BYTES <= NWSLOT * WSLOT_BYTES, "extra page buffers exceed the weight ring");

// The tensor-core page loop (a.tc) copies pages as 128-byte swizzled TMA
// boxes, whose destination must sit on a 1024-byte boundary: its 16 buffers
// start at the first such boundary of the dynamic shared memory (weight-ring
// and activation regions, idle then: a.tc is set only in programs without
// small-batch GEMV stages), followed by its attention scratch and the
// per-warp states of both heads.
constexpr int ATT_TC_SM_OFF = ATT_NBUF_MAX * ATT_PAGE_BYTES + 1024;
constexpr int ATT_TC_COMB_OFF = ATT_TC_SM_OFF + 2048;
static_assert(ATT_TC_COMB_OFF + NWARPS * 2 * (HD + 2) * 4 <= SM_R_OFF, "tensor-core attention region");
QTB_DEV char *att_tc_buf(char *smem, int i) {
  return smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u) + i * ATT_PAGE_BYTES;
}

// Page buffer i (of a.nbuf): the first ATT_NBUF follow the attention scratch
// in the activation region; the others take the weight-ring region, which is
// idle in a program without small-batch GEMV stages.
QTB_DEV uint16_t *att_buf(char *smem, int i) {
  return reinterpret_cast<uint16_t *>(i < ATT_NBUF ? smem + SM_X_OFF + 2048 + i * ATT_PAGE_BYTES
                                                   : smem + SM_W_OFF + (i - ATT_NBUF) * ATT_PAGE_BYTES);
}

struct AttnItem {
  int b, g, sp, pos, L, npages, nsp, p_begin, p_end;
  bool bad_pos;
};

// The attention scratch of a stage (where the tensor-core loop keeps it, or
// at the start of the activation region).
QTB_DEV AttnSmem *attn_sm(const AttnArgs &a, char *smem) {
  return reinterpret_cast<AttnSmem *>(smem + (a.tc ? ATT_TC_SM_OFF : SM_X_OFF));
}

// Pages per split for a sequence of np pages: at least min_pps, at most
// max_splits splits.
QTB_DEV int attn_pps(const AttnArgs &a, int np) {
  const int nsp = max(1, min(a.max_splits, (np + a.min_pps - 1) / a.min_pps));
  return (np + nsp - 1) / nsp;
}

// 1 / sqrt(a) of the per-head QK RMSNorm (a = mean of squares + eps > 0).
// With `tab` it follows the reference's x86 build of qwen_rms_norm_per_head
// (qwen_tts_kernels.c:486-577 compiled with -O3 -ffast-math, which lowers
// 1.0f / sqrtf(x) to an rsqrtss seed x0 and one Newton step
// (x0 a x0 - 3) (-x0 / 2), with that FMA): tab holds the host CPU's rsqrtss
// result for every input in [1, 4) at 12 leading mantissa bits (the seed
// depends only on those and the exponent's parity, and scales exactly by
// powers of 4; checked on the host when the table is built), so the K/V bytes
// this engine appends equal the reference's on that host.  Without a table (or
// for a subnormal a) it is IEEE 1 / sqrtf.
QTB_DEV float qk_inv_rms(float a, const unsigned *tab) {
  const unsigned u = __float_as_uint(a);
  if (!tab || u < 0x00800000u || u >= 0x7f800000u) return 1.0f / sqrtf(a);
  const int e = (int)(u >> 23) - 127, par = e & 1;
  const unsigned seed = __ldg(tab + (((unsigned)par << 12) | ((u >> 11) & 0xfffu)));
  const float x0 = __uint_as_float(seed - ((unsigned)((e - par) / 2) << 23));
  const float t = __fmul_rn(x0, a);
  return __fmul_rn(__fmaf_rn(t, x0, -3.0f), __fmul_rn(x0, -0.5f));
}

// Warp-wide: the prologue values of one 128-dim row of slot b's QKV output at
// position pos -- which = 0, 1: query head 2g + which; 2: key head g; 3: value
// head g -- with the per-head QK RMSNorm and RoPE applied to q and k.  Lane j
// holds dims j, j + 32, j + 64, j + 96.
QTB_DEV void attn_row(const AttnArgs &a, int b, int g, int which, int pos, int lane, float v[4]) {
  const int q_dim = a.n_heads * HD, kv_dim = a.n_kv * HD;
  const float *src;
  const float *nw = nullptr;
  if (which < 2) { src = a.qkv + (size_t)b * a.ld_qkv + (2 * g + which) * HD; nw = a.q_norm; }
  else if (which == 2) { src = a.qkv + (size_t)b * a.ld_qkv + q_dim + g * HD; nw = a.k_norm; }
  else src = a.qkv + (size_t)b * a.ld_qkv + q_dim + kv_dim + g * HD;
  float gw[4], rc[2], rs[2];
#pragma unroll
  for (int i = 0; i < 4; i++) v[i] = __ldcg(src + lane + 32 * i);
  if (nw) {   // independent of the row values: issue with them
#pragma unroll
    for (int i = 0; i < 4; i++) gw[i] = __ldg(nw + lane + 32 * i);
#pragma unroll
    for (int i = 0; i < 2; i++) {
      rc[i] = __ldg(a.rope_cos + (size_t)pos * (HD / 2) + lane + 32 * i);
      rs[i] = __ldg(a.rope_sin + (size_t)pos * (HD / 2) + lane + 32 * i);
    }
  }
  if (nw) {
    // the reference's per-head RMSNorm in its x86 build's operation order
    // (qwen_rms_norm_per_head, qwen_tts_kernels.c:486-577): sixteen-lane
    // FMA accumulators over dims j, j+32, j+64, j+96 (lane j) and j+16, ...
    // (lane j+16) -- this lane's own four values -- then the pairwise tree
    // (+16, +8, +4, +2, +1); mean + eps as one FMA; x * w * inv
    float ss = __fmul_rn(v[0], v[0]);
    ss = __fmaf_rn(v[1], v[1], ss);
    ss = __fmaf_rn(v[2], v[2], ss);
    ss = __fmaf_rn(v[3], v[3], ss);
    ss = warp_sum(ss);
    const float inv = qk_inv_rms(__fmaf_rn(ss, 1.0f / (float)HD, a.eps), a.rsq_tab);
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = __fmul_rn(__fmul_rn(v[i], gw[i]), inv);
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const float c = rc[i], s = rs[i];
      const float x1 = v[i], x2 = v[i + 2];
      v[i] = fmaf(x1, c, -(x2 * s));
      v[i + 2] = fmaf(x2, c, x1 * s);
    }
  }
}

// Decode work item -> (slot, kv head, split) and the split's page range.
// Returns false for items beyond the slot's split count (or a bad position).
QTB_DEV bool attn_item(const AttnArgs &a, int item, AttnItem &it) {
  it.bad_pos = false;
  it.sp = item % a.max_splits;
  const int bg = item / a.max_splits;
  it.g = bg % a.n_kv;
  it.b = bg / a.n_kv;
  it.pos = a.pos_ptr ? __ldcg(a.pos_ptr + it.b) : a.pos_const;
  if (it.pos < 0 || it.pos >= a.rope_len || it.pos >= a.pt_stride * PAGE) { it.bad_pos = true; return false; }
  it.L = it.pos + 1;
  it.npages = (it.L + PAGE - 1) / PAGE;
  const int pps = attn_pps(a, it.npages);
  it.nsp = (it.npages + pps - 1) / pps;
  if (it.sp >= it.nsp) return false;
  it.p_begin = it.sp * pps;
  it.p_end = min(it.npages, it.p_begin + pps);
  return true;
}

// Warp-wide, dynamic order: items of batch slot b are pre[b] .. pre[b+1]-1
// (KV head major, then split); pre[B] = items in all.  Returns that count, or
// -1 for a position outside the cache (nothing written then).
QTB_DEV int attn_prefix(const AttnArgs &a, int B, AttnSmem *sm) {
  const int lane = threadIdx.x & 31;
  int run = 0;
  bool bad = false;
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    int cnt = 0;
    if (b < B) {
      const int pos = a.pos_ptr ? __ldcg(a.pos_ptr + b) : a.pos_const;
      if (pos < 0 || pos >= a.rope_len || pos >= a.pt_stride * PAGE) {
        bad = true;
      } else {
        const int np = (pos + PAGE) / PAGE;
        const int pps = attn_pps(a, np);
        cnt = a.n_kv * ((np + pps - 1) / pps);
      }
    }
    int v = cnt;   // inclusive scan over the lanes
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (b < B) sm->pre[b] = run + v - cnt;
    run += __shfl_sync(0xffffffffu, v, 31);
  }
  if (__any_sync(0xffffffffu, bad)) return -1;
  if (lane == 0) sm->pre[B] = run;
  __syncwarp();
  return run;
}

// Dynamic-order item -> (slot, kv head, split); item < pre[B].
QTB_DEV void attn_item_dyn(const AttnArgs &a, int B, int item, const AttnSmem *sm, AttnItem &it) {
  int lo = 0, hi = B;   // pre[lo] <= item < pre[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (sm->pre[mid] <= item) lo = mid; else hi = mid;
  }
  it.bad_pos = false;
  it.b = lo;
  const int r = item - sm->pre[lo];
  const int nsp = (sm->pre[lo + 1] - sm->pre[lo]) / a.n_kv;
  it.g = r / nsp;
  it.sp = r - it.g * nsp;
  it.pos = a.pos_ptr ? __ldcg(a.pos_ptr + it.b) : a.pos_const;
  it.L = it.pos + 1;
  it.npages = (it.L + PAGE - 1) / PAGE;
  const int pps = attn_pps(a, it.npages);
  it.nsp = nsp;
  it.p_begin = it.sp * pps;
  it.p_end = min(it.npages, it.p_begin + pps);
}

// Take the next work item of a dynamic attention stage (one thread).
QTB_DEV int attn_take(KCtx &kc) { return (int)(atomicAdd(&kc.ctl->att_work, 1u) - kc.att_base); }

// Bulk-copy pool page `page` of KV head g into the ring buffer of stream
// position ctr (one thread; the caller records kc.att_issued).
QTB_DEV void attn_issue_pg(const AttnArgs &a, int page, int g, unsigned ctr, KCtx &kc, char *smem) {
  const int nb = a.nbuf;
  const int buf = ctr % nb;
  if (page < 0 || page >= a.n_pages) { raise_err(kc, ERR_BAD_PAGE, page); page = 0; }
  if (a.tc) {
    // K dims 0-63, 64-127, then V: four 16 x 64 boxes of 2 KB, swizzled
    char *dst = att_tc_buf(smem, buf);
    const int y = (page * a.n_kv + g) * PAGE;
    mbar_arrive_expect_tx(kc.bars + buf, ATT_PAGE_BYTES);
    tma_load_3d(dst, a.kmap, 0, y, a.layer, kc.bars + buf);
    tma_load_3d(dst + 2048, a.kmap, 64, y, a.layer, kc.bars + buf);
    tma_load_3d(dst + 4096, a.vmap, 0, y, a.layer, kc.bars + buf);
    tma_load_3d(dst + 6144, a.vmap, 64, y, a.layer, kc.bars + buf);
    return;
  }
  uint16_t *dstk = att_buf(smem, buf);
  const size_t off = (((size_t)page * a.n_kv + g) * PAGE) * HD;
  mbar_arrive_expect_tx(kc.bars + buf, ATT_PAGE_BYTES);
  bulk_g2s(dstk, a.kpool + off, PAGE * HD * 2, kc.bars + buf);
  bulk_g2s(dstk + PAGE * HD, a.vpool + off, PAGE * HD * 2, kc.bars + buf);
}
// ... page i of the item's range.
QTB_DEV void attn_issue1(const AttnArgs &a, const AttnItem &it, int i, unsigned ctr, KCtx &kc, char *smem) {
  attn_issue_pg(a, __ldg(a.page_table + (size_t)it.b * a.pt_stride + it.p_begin + i), it.g, ctr, kc, smem);
}

// Warp-wide: bulk-copy pages [i0, i1) (i1 - i0 <= 32) of the item, one per lane.
QTB_DEV void attn_issue(const AttnArgs &a, const AttnItem &it, int i0, int i1, KCtx &kc, char *smem) {
  const int lane = threadIdx.x & 31;
  if (i0 >= i1) return;
  if (lane < i1 - i0) {
    // the buffers were last touched through the generic proxy
    asm volatile("fence.proxy.async;" ::: "memory");
    attn_issue1(a, it, i0 + lane, kc.page_ctr + i0 + lane, kc, smem);
  }
  __syncwarp();
  if (lane == 0) kc.att_issued = kc.page_ctr + i1;
  __syncwarp();
}

// Warp 0, before the grid barrier: take this CTA's first item of the coming
// attention stage and bulk-copy its first pages (older positions only; the
// newest token is patched in from registers by the stage itself).
QTB_CALL void attn_prefetch(const AttnArgs &a, int B, KCtx &kc, char *smem) {
  const int lane = threadIdx.x & 31;
  AttnSmem *sm = attn_sm(a, smem);
  AttnItem it;
  if (a.dyn) {
    const int tot = attn_prefix(a, B, sm);
    if (tot < 0) return;   // the stage reports it
    int item = 0;
    if (lane == 0) item = attn_take(kc);
    item = __shfl_sync(0xffffffffu, item, 0);
    if (lane == 0) { kc.att_first = item; kc.att_tot = tot; }
    __syncwarp();
    if (item >= tot) return;
    attn_item_dyn(a, B, item, sm, it);
  } else {
    const int n_items = B * a.n_kv * a.max_splits;
    if ((int)blockIdx.x >= n_items || !attn_item(a, blockIdx.x, it)) return;
  }
  const int n = min(it.p_end - it.p_begin, a.nbuf);
  if (lane == 0) kc.att_nbuf = a.nbuf;
  attn_issue(a, it, 0, n, kc, smem);
}

// Tensor-core pages of one decode attention item (large batches).  Warp w
// takes the item's pages w, w + 16, ... and w + 8, w + 24, ..., two per step
// (independent chains sharing one softmax update), with both query heads of
// the GQA group at once, on the bf16 MMA (m16n8k16, f32 accumulate):
//  - scores S[16 tokens x 8] = K[16 x 128] q^T, the 8 MMA columns being
//    (part p, head h) = 2 p + h: q carried as three bf16 parts (24 bits).  The
//    K rows come from the swizzled page (lane: row gid, 16-byte chunk 2 tig +
//    (j & 1) of box j >> 1 per step pair j; the MMA's k order follows that
//    dimension order, and q's fragments use the same one), in two chains;
//  - the online softmax of each head over the pages' tokens (reference
//    recurrence of qwen_causal_attention_bf16kv, per step);
//  - O^T[128 x (p, h)] += V^T[128 x 16 tokens] P^T: A = V^T from
//    ldmatrix.trans on the swizzled V box (conflict-free), B = the three bf16
//    parts of the f32 probabilities, rebuilt from the score layout with four
//    shuffles; all four accumulator registers of a tile are used.
// The warp's per-head state (max, sum, 128 outputs) goes to s_acc / s_ml
// ([NWARPS][2][HD], [NWARPS][2][2]).  Returns false after a failed wait.
__device__ __noinline__ bool attn_pages_tc(const AttnArgs &a, const AttnItem &it, const AttnItem &nx, int nx_n,
                                           bool owns_new, KCtx &kc, char *smem_base, const AttnSmem *sm,
                                           float *s_acc, float *s_ml) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int NB = a.nbuf;
  const int n = it.p_end - it.p_begin;
  const int *pt = a.page_table + (size_t)it.b * a.pt_stride;
  const int hq = gid & 1, pq = gid >> 1;   // this lane's MMA column / P row: head, part
  // q fragments (B operand of the score MMAs)
  uint32_t qf[4][4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const float *q = sm->q[hq] + (j >> 1) * 64 + (2 * tig + (j & 1)) * 8;
#pragma unroll
    for (int u = 0; u < 4; u++) qf[j][u] = gid < 6 ? split_pack<false>(q[2 * u], q[2 * u + 1], pq) : 0u;
  }
  float m_w[2] = {-INFINITY, -INFINITY}, l_w[2] = {0.f, 0.f};
  // O^T tile m: dims 16 m + gid (0, 1) and 16 m + gid + 8 (2, 3), columns
  // (part tig, head 0 / 1)
  float oacc[8][4];
#pragma unroll
  for (int m = 0; m < 8; m++) oacc[m][0] = oacc[m][1] = oacc[m][2] = oacc[m][3] = 0.f;
  bool ok = true;
  // the scores of one page: two independent chains (dims 0-63, 64-127), parts summed
  auto scores = [&](const char *pg_k, float (&sc)[4]) {
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const char *kb = pg_k + (j >> 1) * 2048;
      const int cc = ((2 * tig + (j & 1)) ^ (gid & 7)) << 4;
      const uint4 w0 = *reinterpret_cast<const uint4 *>(kb + gid * 128 + cc);
      const uint4 w1 = *reinterpret_cast<const uint4 *>(kb + (gid + 8) * 128 + cc);
      const uint32_t A0[4] = {w0.x, w1.x, w0.y, w1.y};
      const uint32_t A1[4] = {w0.z, w1.z, w0.w, w1.w};
      if (j < 2) {
        mma_bf16(s0, A0, qf[j][0], qf[j][1]);
        mma_bf16(s0, A1, qf[j][2], qf[j][3]);
      } else {
        mma_bf16(s1, A0, qf[j][0], qf[j][1]);
        mma_bf16(s1, A1, qf[j][2], qf[j][3]);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; e++) {
      sc[e] = s0[e] + s1[e];
      sc[e] += __shfl_xor_sync(0xffffffffu, sc[e], 1);
      sc[e] += __shfl_xor_sync(0xffffffffu, sc[e], 2);
    }
  };
  // P^T fragments (tokens x (part, head)) of one page from its probabilities
  // in the score layout: lane (gid, tig) holds P[gid][2 tig, 2 tig + 1] in pb[0]
  // and P[gid][2 tig + 8, 2 tig + 9] in pb[1]
  auto pfrag = [&](const float (&pr)[4], uint32_t (&pb)[2]) {
    const float off1 = (tig & 1) ? pr[1] : pr[0], off2 = (tig & 1) ? pr[3] : pr[2];
    const int sa = (2 * tig) * 4 + hq, sb = (2 * tig + 1) * 4 + hq;
    const float pa = __shfl_sync(0xffffffffu, off1, sa), p2 = __shfl_sync(0xffffffffu, off1, sb);
    const float pc = __shfl_sync(0xffffffffu, off2, sa), pd = __shfl_sync(0xffffffffu, off2, sb);
    pb[0] = gid < 6 ? split_pack<false>(pa, p2, pq) : 0u;
    pb[1] = gid < 6 ? split_pack<false>(pc, pd, pq) : 0u;
  };
  // the newest token comes from shared memory (its copy may predate the append)
  auto patch = [&](char *pg_k) {
    const int row = it.pos % PAGE, c = lane & 15;
    const uint16_t *src = (lane < 16 ? sm->knew : sm->vnew) + c * 8;
    char *dst = pg_k + (lane < 16 ? 0 : 4096) + (c >> 3) * 2048 + row * 128 + (((c & 7) ^ (row & 7)) << 4);
    *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
    __syncwarp();
  };
  // Pages i and i + NWARPS per step: the two pages' chains are independent
  // and share one softmax update.
  for (int i = warp; i < n; i += 2 * NWARPS) {
    const int i2 = i + NWARPS;
    const bool two = i2 < n;
    const unsigned ctr = kc.page_ctr + i, ctr2 = ctr + NWARPS;
    const int buf = ctr % NB, buf2 = ctr2 % NB;
    bool landed = mbar_wait(kc.bars + buf, (ctr / NB) & 1u, WAIT_LIMIT_CYCLES);
    if (two) landed = mbar_wait(kc.bars + buf2, (ctr2 / NB) & 1u, WAIT_LIMIT_CYCLES) && landed;
    if (!__all_sync(0xffffffffu, landed)) {
      if (lane == 0) raise_err(kc, ERR_MBAR_TIMEOUT, i);
      ok = false;
      break;
    }
    char *pk1 = att_tc_buf(smem_base, buf), *pk2 = att_tc_buf(smem_base, buf2);
    const int pg = it.p_begin + i, pg2 = it.p_begin + i2;
    const int ntok = min(PAGE, it.L - pg * PAGE), ntok2 = two ? min(PAGE, it.L - pg2 * PAGE) : 0;
    if (owns_new && pg == it.npages - 1) patch(pk1);
    if (owns_new && two && pg2 == it.npages - 1) patch(pk2);
    int refill_page = -1, refill_page2 = -1;
    const int tgt = i + NB, tgt2 = i2 + NB;   // item-relative; >= n: the next item's page tgt - n
    if (lane == 0) {
      if (tgt < n) refill_page = __ldg(pt + it.p_begin + tgt);
      else if (tgt - n < nx_n) refill_page = __ldg(a.page_table + (size_t)nx.b * a.pt_stride + nx.p_begin + (tgt - n));
      if (two) {
        if (tgt2 < n) refill_page2 = __ldg(pt + it.p_begin + tgt2);
        else if (tgt2 - n < nx_n)
          refill_page2 = __ldg(a.page_table + (size_t)nx.b * a.pt_stride + nx.p_begin + (tgt2 - n));
      }
    }
    float sc1[4], sc2[4] = {0.f, 0.f, 0.f, 0.f};
    scores(pk1, sc1);
    if (two) scores(pk2, sc2);
    // sc: tokens gid (e = 0, 1) and gid + 8 (e = 2, 3) of head e & 1
    const bool va = gid < ntok, vb = gid + 8 < ntok, vc = gid < ntok2, vd = gid + 8 < ntok2;
    float pr1[4], pr2[4], corr[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const float x0 = va ? sc1[h] * a.scale : -INFINITY, x1 = vb ? sc1[2 + h] * a.scale : -INFINITY;
      const float y0 = vc ? sc2[h] * a.scale : -INFINITY, y1 = vd ? sc2[2 + h] * a.scale : -INFINITY;
      float mx = fmaxf(fmaxf(x0, x1), fmaxf(y0, y1));
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_w[h], mx);   // finite: token 0 of every page is valid
      corr[h] = (m_w[h] == -INFINITY) ? 0.f : expf(m_w[h] - m_new);
      pr1[h] = va ? expf(x0 - m_new) : 0.f;
      pr1[2 + h] = vb ? expf(x1 - m_new) : 0.f;
      pr2[h] = vc ? expf(y0 - m_new) : 0.f;
      pr2[2 + h] = vd ? expf(y1 - m_new) : 0.f;
      l_w[h] = l_w[h] * corr[h] + ((pr1[h] + pr1[2 + h]) + (pr2[h] + pr2[2 + h]));
      m_w[h] = m_new;
    }
#pragma unroll
    for (int m = 0; m < 8; m++) {
      oacc[m][0] *= corr[0];
      oacc[m][1] *= corr[1];
      oacc[m][2] *= corr[0];
      oacc[m][3] *= corr[1];
    }
    uint32_t pb1[2], pb2[2];
    pfrag(pr1, pb1);
    pfrag(pr2, pb2);   // zeros for a missing second page
    // ---- O^T += V^T P^T: A = V^T (ldmatrix.trans of the swizzled V box),
    // B = P^T; matrix j of a tile: tokens 8 (j >> 1) .., dims 16 m + 8 (j & 1) ..
    const int mj = lane >> 3, r = lane & 7;
    const int tok = r + 8 * (mj >> 1);
#pragma unroll
    for (int m = 0; m < 8; m++) {
      const int c = 2 * m + (mj & 1);
      const int off = 4096 + (c >> 3) * 2048 + tok * 128 + (((c & 7) ^ r) << 4);
      uint32_t va4[4];
      ldsm_x4_trans(va4, pk1 + off);
      mma_bf16(oacc[m], va4, pb1[0], pb1[1]);
      if (two) {
        ldsm_x4_trans(va4, pk2 + off);
        mma_bf16(oacc[m], va4, pb2[0], pb2[1]);
      }
    }
    // the warp is done with both buffers: refill each with its stream position + NB
    __syncwarp();
    if (lane == 0) {
      const bool r1 = tgt < n || tgt - n < nx_n;
      const bool r2 = two && (tgt2 < n || tgt2 - n < nx_n);
      if (r1 || r2) fence_proxy_async_smem();
      if (r1) attn_issue_pg(a, refill_page, tgt < n ? it.g : nx.g, ctr + NB, kc, smem_base);
      if (r2) attn_issue_pg(a, refill_page2, tgt2 < n ? it.g : nx.g, ctr2 + NB, kc, smem_base);
      if (r1 || r2) atomicMax(&kc.att_issued, (r2 ? ctr2 : ctr) + NB + 1u);
    }
  }
  // ---- the warp's per-head states ----
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) l_w[h] += __shfl_xor_sync(0xffffffffu, l_w[h], o);
#pragma unroll
  for (int m = 0; m < 8; m++)
#pragma unroll
    for (int e = 0; e < 4; e++) {   // the three parts of each head (columns tig = 0, 1, 2; 3 is zero)
      oacc[m][e] += __shfl_xor_sync(0xffffffffu, oacc[m][e], 1);
      oacc[m][e] += __shfl_xor_sync(0xffffffffu, oacc[m][e], 2);
    }
  if (tig == 0) {
    float *d0 = s_acc + (warp * 2) * HD, *d1 = d0 + HD;
#pragma unroll
    for (int m = 0; m < 8; m++) {
      d0[16 * m + gid] = oacc[m][0];
      d1[16 * m + gid] = oacc[m][1];
      d0[16 * m + gid + 8] = oacc[m][2];
      d1[16 * m + gid + 8] = oacc[m][3];
    }
  }
  if (lane < 2) {
    s_ml[(warp * 2 + lane) * 2] = lane ? m_w[1] : m_w[0];
    s_ml[(warp * 2 + lane) * 2 + 1] = lane ? l_w[1] : l_w[0];
  }
  return ok;
}

// The decode attention stage with the tensor-core page loop (a.tc: batch >= 8
// talker stages); same items, prologue and split combine as attn_stage.
__device__ __noinline__ void attn_stage_tc(const AttnArgs &a, int B, char *smem_base, KCtx &kc) {
  char *smem = smem_base + SM_X_OFF;
  AttnSmem *sm = attn_sm(a, smem_base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NB = a.nbuf;

  // ---- this CTA's first item ----
  int n_items, item;
  if (a.dyn) {
    if (kc.att_first < 0) {   // not taken before the barrier
      if (warp == 0) {
        const int tot = attn_prefix(a, B, sm);
        if (lane == 0) {
          sm->flag = tot;
          if (tot >= 0) sm->next = attn_take(kc);
        }
      }
      __syncthreads();
      n_items = sm->flag;
      item = sm->next;
      if (n_items < 0) {
        if (threadIdx.x == 0) raise_err(kc, ERR_BAD_POS, -1);
        return;
      }
    } else {
      n_items = kc.att_tot;
      item = kc.att_first;
    }
  } else {
    n_items = B * a.n_kv * a.max_splits;
    item = blockIdx.x;
  }
  __syncthreads();   // every thread has read the first item before it changes
  if (threadIdx.x == 0) { kc.att_first = -1; kc.att_nbuf = NB; }

  while (item < n_items) {
    AttnItem it;
    if (a.dyn) {
      attn_item_dyn(a, B, item, sm, it);
    } else if (!attn_item(a, item, it)) {
      if (it.bad_pos) {
        if (threadIdx.x == 0) raise_err(kc, ERR_BAD_POS, it.pos);
        return;
      }
      item += gridDim.x;
      continue;
    }
    const int b = it.b, g = it.g, sp = it.sp, pos = it.pos, L = it.L, npages = it.npages, nsp = it.nsp;
    const int p_begin = it.p_begin, p_end = it.p_end;
    // the item that holds the newest page appends the token (decode, append)
    // and patches it into its page buffer from registers (decode only)
    const bool owns_new = (p_end == npages) && a.mode != ATT_ATTEND;
    const int *pt = a.page_table + (size_t)b * a.pt_stride;
    // pages first: the stream positions issued so far are a prefix (the hook
    // before the barrier, or the previous item's refills, may have covered
    // the first ones)
    if (warp == 7 && a.mode != ATT_APPEND) {
      const int done = (int)min(kc.att_issued - kc.page_ctr, (unsigned)NB);
      attn_issue(a, it, done, min(p_end - p_begin, NB), kc, smem_base);
    }
    // dynamic order: take the next item now (the atomic's latency hides behind
    // this one), from a warp that is idle in the prologue
    if (a.dyn && threadIdx.x == 4 * 32) sm->next = attn_take(kc);
    ckpt(kc, 0);

    // ---- prologue: QK RMSNorm + RoPE (+ KV append) ----
    if (warp < 4) {
      float v[4];
      attn_row(a, b, g, warp, pos, lane, v);
      if (warp < 2) {
#pragma unroll
        for (int i = 0; i < 4; i++) sm->q[warp][lane + 32 * i] = v[i];
      } else {
        uint16_t *dst = (warp == 2) ? sm->knew : sm->vnew;
#pragma unroll
        for (int i = 0; i < 4; i++) dst[lane + 32 * i] = (uint16_t)f32_to_bf16_trunc(v[i]);
        if (a.mode == ATT_APPEND && a.pkv) {   // a prefill's prompt K/V, unrounded
          const PromptKV P = *a.pkv;
          const int r = pos - P.p0;
          if (r < 0 || r >= P.cap) {
            if (lane == 0) raise_err(kc, ERR_BAD_POS, pos);
          } else {
            float *dstf = (warp == 2 ? P.k : P.v) + (((size_t)a.layer * a.n_kv + g) * P.cap + r) * HD;
#pragma unroll
            for (int i = 0; i < 4; i++) __stcg(dstf + lane + 32 * i, v[i]);
          }
        }
      }
    }
    __syncthreads();
    if (owns_new && threadIdx.x < 32) {
      const int page = __ldg(pt + pos / PAGE);
      if (page < 0 || page >= a.n_pages) {
        if (threadIdx.x == 0) raise_err(kc, ERR_BAD_PAGE, page);
      } else {
        const int half = threadIdx.x >> 4, part = threadIdx.x & 15;   // 16 x 16 B per K / V row
        uint16_t *pool = half ? a.vpool : a.kpool;
        const uint16_t *srcv = half ? sm->vnew : sm->knew;
        uint4 val = *reinterpret_cast<const uint4 *>(srcv + part * 8);
        uint16_t *dst = pool + (((size_t)page * a.n_kv + g) * PAGE + (pos % PAGE)) * HD + part * 8;
        __stcg(reinterpret_cast<uint4 *>(dst), val);
      }
    }
    if (__syncthreads_or(kc.local_err)) return;
    ckpt(kc, 1);
    const int next = a.dyn ? sm->next : item + (int)gridDim.x;
    if (a.mode == ATT_APPEND) {   // no attention in this stage
      __syncthreads();   // every thread has read sm->next and the new K/V rows
      item = next;
      continue;
    }
    // dynamic order: the next item's pages follow this one's in the stream, so
    // buffers freed near the end of this item already take the next one's
    // pages.  Only from an item of at least NB pages: then the refills cover
    // the next item's first positions without a gap (the issued positions stay
    // a prefix of the stream, which the next item's first issue relies on).
    AttnItem nx;
    int nx_n = 0;
    if (a.dyn && next < n_items && p_end - p_begin >= NB) {
      attn_item_dyn(a, B, next, sm, nx);
      nx_n = nx.p_end - nx.p_begin;
    }

    // ---- main loop over this split's pages ----
    const int n = p_end - p_begin;
    const int tid = threadIdx.x;
    const int hh = tid >> 7, d = tid & 127;
    float Mh = -INFINITY, Lh = 0.f, acc = 0.f;
    {
      // tensor-core pages: per-warp states of both heads, combined in warp order
      float *s_acc = reinterpret_cast<float *>(smem_base + ATT_TC_COMB_OFF);   // [NWARPS][2][HD]
      float *s_ml = s_acc + NWARPS * 2 * HD;                                    // [NWARPS][2][2]
      attn_pages_tc(a, it, nx, nx_n, owns_new, kc, smem_base, sm, s_acc, s_ml);
      if (__syncthreads_or(kc.local_err)) return;   // copies still in flight are drained on the way out
      if (tid == 0) kc.page_ctr += n;
#pragma unroll
      for (int w = 0; w < NWARPS; w++) Mh = fmaxf(Mh, s_ml[(w * 2 + hh) * 2]);
#pragma unroll
      for (int w = 0; w < NWARPS; w++) {
        const float mw = s_ml[(w * 2 + hh) * 2];
        const float e = (mw == -INFINITY) ? 0.f : expf(mw - Mh);
        Lh += s_ml[(w * 2 + hh) * 2 + 1] * e;
        acc += s_acc[(w * 2 + hh) * HD + d] * e;
      }
    }
    ckpt(kc, 2);

    // ---- output / split combine ----
    const int head = 2 * g + hh;
    if (nsp == 1) {
      __stcg(a.out + (size_t)b * a.ld_out + head * HD + d, acc * (1.0f / Lh));
    } else {
      float *wsi = a.ws + ((((size_t)b * a.n_kv + g) * a.max_splits + sp) * 2 + hh) * (HD + 2);
      __stcg(wsi + d, acc);
      if (d == 0) { __stcg(wsi + HD, Mh); __stcg(wsi + HD + 1, Lh); }
      __threadfence();
      __syncthreads();
      if (tid == 0) sm->flag = (atomicAdd(a.sem + (size_t)b * a.n_kv + g, 1u) == (unsigned)(nsp - 1));
      __syncthreads();
      if (sm->flag) {
        __threadfence();
        const float *w0 = a.ws + ((((size_t)b * a.n_kv + g) * a.max_splits) * 2 + hh) * (HD + 2);
        float M = -INFINITY;
        for (int s2 = 0; s2 < nsp; s2++) M = fmaxf(M, __ldcg(w0 + (size_t)s2 * 2 * (HD + 2) + HD));
        float Ls = 0.f, O = 0.f;
        for (int s2 = 0; s2 < nsp; s2++) {
          const float *wsp = w0 + (size_t)s2 * 2 * (HD + 2);
          const float e = expf(__ldcg(wsp + HD) - M);
          Ls += __ldcg(wsp + HD + 1) * e;
          O += __ldcg(wsp + d) * e;
        }
        __stcg(a.out + (size_t)b * a.ld_out + head * HD + d, O * (1.0f / Ls));
        if (tid == 0) a.sem[(size_t)b * a.n_kv + g] = 0u;
      }
    }
    __syncthreads();
    item = next;
  }
  // every CTA took exactly one item past the end: the counter now stands at
  // the next dynamic stage's base
  if (a.dyn && threadIdx.x == 0) kc.att_base += (unsigned)n_items + gridDim.x;
}

__device__ __noinline__ void attn_stage(const AttnArgs &a, int B, char *smem_base, KCtx &kc) {
  if (a.tc) {
    attn_stage_tc(a, B, smem_base, kc);
    return;
  }
  char *smem = smem_base + SM_X_OFF;
  AttnSmem *sm = reinterpret_cast<AttnSmem *>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NB = a.nbuf;

  // ---- this CTA's first item ----
  int n_items, item;
  if (a.dyn) {
    if (kc.att_first < 0) {   // not taken before the barrier
      if (warp == 0) {
        const int tot = attn_prefix(a, B, sm);
        if (lane == 0) {
          sm->flag = tot;
          if (tot >= 0) sm->next = attn_take(kc);
        }
      }
      __syncthreads();
      n_items = sm->flag;
      item = sm->next;
      if (n_items < 0) {
        if (threadIdx.x == 0) raise_err(kc, ERR_BAD_POS, -1);
        return;
      }
    } else {
      n_items = kc.att_tot;
      item = kc.att_first;
    }
  } else {
    n_items = B * a.n_kv * a.max_splits;
    item = blockIdx.x;
  }
  __syncthreads();   // every thread has read the first item before it changes
  if (threadIdx.x == 0) { kc.att_first = -1; kc.att_nbuf = NB; }

  while (item < n_items) {
    AttnItem it;
    if (a.dyn) {
      attn_item_dyn(a, B, item, sm, it);
    } else if (!attn_item(a, item, it)) {
      if (it.bad_pos) {
        if (threadIdx.x == 0) raise_err(kc, ERR_BAD_POS, it.pos);
        return;
      }
      item += gridDim.x;
      continue;
    }
    const int b = it.b, g = it.g, sp = it.sp, pos = it.pos, L = it.L, npages = it.npages, nsp = it.nsp;
    const int p_begin = it.p_begin, p_end = it.p_end;
    // the item that holds the newest page appends the token (decode, append)
    // and patches it into its page buffer from registers (decode only)
    const bool owns_new = (p_end == npages) && a.mode != ATT_ATTEND;
    const int *pt = a.page_table + (size_t)b * a.pt_stride;
    // pages first: the stream positions issued so far are a prefix (the hook
    // before the barrier, or the previous item's refills, may have covered
    // the first ones)
    if (warp == 7 && a.mode != ATT_APPEND) {
      const int done = (int)min(kc.att_issued - kc.page_ctr, (unsigned)NB);
      attn_issue(a, it, done, min(p_end - p_begin, NB), kc, smem_base);
    }
    // dynamic order: take the next item now (the atomic's latency hides behind
    // this one), from a warp that is idle in the prologue
    if (a.dyn && threadIdx.x == 4 * 32) sm->next = attn_take(kc);
    ckpt(kc, 0);

    // ---- prologue: QK RMSNorm + RoPE (+ KV append) ----
    if (warp < 4) {
      float v[4];
      attn_row(a, b, g, warp, pos, lane, v);
      if (warp < 2) {
#pragma unroll
        for (int i = 0; i < 4; i++) sm->q[warp][lane + 32 * i] = v[i];
      } else {
        uint16_t *dst = (warp == 2) ? sm->knew : sm->vnew;
#pragma unroll
        for (int i = 0; i < 4; i++) dst[lane + 32 * i] = (uint16_t)f32_to_bf16_trunc(v[i]);
        if (a.mode == ATT_APPEND && a.pkv) {   // a prefill's prompt K/V, unrounded
          const PromptKV P = *a.pkv;
          const int r = pos - P.p0;
          if (r < 0 || r >= P.cap) {
            if (lane == 0) raise_err(kc, ERR_BAD_POS, pos);
          } else {
            float *dstf = (warp == 2 ? P.k : P.v) + (((size_t)a.layer * a.n_kv + g) * P.cap + r) * HD;
#pragma unroll
            for (int i = 0; i < 4; i++) __stcg(dstf + lane + 32 * i, v[i]);
          }
        }
      }
    }
    __syncthreads();
    if (owns_new && threadIdx.x < 32) {
      const int page = __ldg(pt + pos / PAGE);
      if (page < 0 || page >= a.n_pages) {
        if (threadIdx.x == 0) raise_err(kc, ERR_BAD_PAGE, page);
      } else {
        const int half = threadIdx.x >> 4, part = threadIdx.x & 15;   // 16 x 16 B per K / V row
        uint16_t *pool = half ? a.vpool : a.kpool;
        const uint16_t *srcv = half ? sm->vnew : sm->knew;
        uint4 val = *reinterpret_cast<const uint4 *>(srcv + part * 8);
        uint16_t *dst = pool + (((size_t)page * a.n_kv + g) * PAGE + (pos % PAGE)) * HD + part * 8;
        __stcg(reinterpret_cast<uint4 *>(dst), val);
      }
    }
    if (__syncthreads_or(kc.local_err)) return;
    ckpt(kc, 1);
    const int next = a.dyn ? sm->next : item + (int)gridDim.x;
    if (a.mode == ATT_APPEND) {   // no attention in this stage
      __syncthreads();   // every thread has read sm->next and the new K/V rows
      item = next;
      continue;
    }
    // dynamic order: the next item's pages follow this one's in the stream, so
    // buffers freed near the end of this item already take the next one's
    // pages.  Only from an item of at least NB pages: then the refills cover
    // the next item's first positions without a gap (the issued positions stay
    // a prefix of the stream, which the next item's first issue relies on).
    AttnItem nx;
    int nx_n = 0;
    if (a.dyn && next < n_items && p_end - p_begin >= NB) {
      attn_item_dyn(a, B, next, sm, nx);
      nx_n = nx.p_end - nx.p_begin;
    }

    // ---- main loop over this split's pages ----
    // Warp w handles head h = w & 1 of the item's pages i = w / 2 (mod 4), so
    // four pages are in work at once, each by the two warps of its GQA group;
    // every warp keeps its own online softmax (running max m, sum l, output
    // dims 4 lane .. 4 lane + 3), combined across warps in warp order at the
    // end.  The split of pages among warps depends on the item alone, so the
    // result does not depend on which CTA ran it.  Page i sits in ring buffer
    // (stream position) % NB; once both warps of the pair are done with a
    // buffer (named barrier per pair) the head-0 warp refills it with stream
    // position + NB (this item's page i + NB, or a page of the next item).
    const int n = p_end - p_begin;
    const int tid = threadIdx.x;
    const int h = warp & 1, pw = warp >> 1;
    const int t = lane & 15, half = lane >> 4;
    float m_w = -INFINITY, l_w = 0.f, acc4[4] = {0.f, 0.f, 0.f, 0.f};
    // With 16 buffers a pair takes two of its pages per step (i and i + 4):
    // the two pages' dot products and P.V run as independent chains and share
    // one softmax update; with 4 buffers (small batches) one page per step.
    float acc4b[4] = {0.f, 0.f, 0.f, 0.f};
    if (NB >= 2 * (NWARPS / 2)) {
      for (int i = pw; i < n; i += 2 * (NWARPS / 2)) {
        const int i2 = i + NWARPS / 2;
        const bool two = i2 < n;
        const unsigned ctr = kc.page_ctr + i, ctr2 = ctr + NWARPS / 2;
        const int buf = ctr % NB, buf2 = ctr2 % NB;
        // every lane observes the phase flips, which makes the bulk-copied bytes
        // visible to it; the pair agrees on the outcome (named barrier 1 + pw),
        // so a timeout ends both warps' loops at the same page
        bool landed = mbar_wait(kc.bars + buf, (ctr / NB) & 1u, WAIT_LIMIT_CYCLES);
        if (two) landed = mbar_wait(kc.bars + buf2, (ctr2 / NB) & 1u, WAIT_LIMIT_CYCLES) && landed;
        if (!bar_and_n(1 + pw, 64, landed)) {
          if (lane == 0 && !landed) raise_err(kc, ERR_MBAR_TIMEOUT, i);
          break;
        }
        uint16_t *kb = att_buf(smem_base, buf);
        uint16_t *vb = kb + PAGE * HD;
        uint16_t *kb2 = att_buf(smem_base, buf2);
        uint16_t *vb2 = kb2 + PAGE * HD;
        const int ntok = min(PAGE, L - (p_begin + i) * PAGE);
        const int ntok2 = two ? min(PAGE, L - (p_begin + i2) * PAGE) : 0;
        if (owns_new && (p_begin + i == npages - 1 || (two && p_begin + i2 == npages - 1))) {
          // the newest token comes from shared memory, not from the copy (both
          // warps of the page write the same bytes)
          const int slot = pos % PAGE;
          uint16_t *kp = (p_begin + i == npages - 1) ? kb : kb2;
          uint16_t *vp = kp + PAGE * HD;
          *reinterpret_cast<uint2 *>(kp + slot * HD + 4 * lane) = *reinterpret_cast<const uint2 *>(sm->knew + 4 * lane);
          *reinterpret_cast<uint2 *>(vp + slot * HD + 4 * lane) = *reinterpret_cast<const uint2 *>(sm->vnew + 4 * lane);
          __syncwarp();
        }
        // the pages that will reuse these buffers: their indices are loaded
        // now, so the refills at the end of the step do not wait for them
        int refill_page = -1, refill_page2 = -1;
        if (h == 0 && lane == 0) {
          const int tgt = i + NB, tgt2 = i2 + NB;
          if (tgt < n) refill_page = __ldg(pt + p_begin + tgt);
          else if (tgt - n < nx_n) refill_page = __ldg(a.page_table + (size_t)nx.b * a.pt_stride + nx.p_begin + (tgt - n));
          if (two) {
            if (tgt2 < n) refill_page2 = __ldg(pt + p_begin + tgt2);
            else if (tgt2 - n < nx_n) refill_page2 = __ldg(a.page_table + (size_t)nx.b * a.pt_stride + nx.p_begin + (tgt2 - n));
          }
        }
        // scores of both pages, as in the one-page loop; the q reads are shared
        const float *qh = sm->q[h] + half * 64;
        float sdot, sdot2 = 0.f;
        {
          float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
          const uint16_t *kr = kb + t * HD + half * 64;
          if (two) {
            float u0 = 0.f, u1 = 0.f, u2 = 0.f, u3 = 0.f;
            const uint16_t *kr2 = kb2 + t * HD + half * 64;
  #pragma unroll
            for (int jj = 0; jj < 8; jj++) {
              const int jq = (jj + t) & 7;
              const uint4 kk = *reinterpret_cast<const uint4 *>(kr + 8 * jq);
              const uint4 k2 = *reinterpret_cast<const uint4 *>(kr2 + 8 * jq);
              const float4 qa = *reinterpret_cast<const float4 *>(qh + 8 * jq);
              const float4 qb = *reinterpret_cast<const float4 *>(qh + 8 * jq + 4);
              s0 = fmaf(qa.x, bf16lo(kk.x), s0);
              s1 = fmaf(qa.y, bf16hi(kk.x), s1);
              s2 = fmaf(qa.z, bf16lo(kk.y), s2);
              s3 = fmaf(qa.w, bf16hi(kk.y), s3);
              u0 = fmaf(qa.x, bf16lo(k2.x), u0);
              u1 = fmaf(qa.y, bf16hi(k2.x), u1);
              u2 = fmaf(qa.z, bf16lo(k2.y), u2);
              u3 = fmaf(qa.w, bf16hi(k2.y), u3);
              s0 = fmaf(qb.x, bf16lo(kk.z), s0);
              s1 = fmaf(qb.y, bf16hi(kk.z), s1);
              s2 = fmaf(qb.z, bf16lo(kk.w), s2);
              s3 = fmaf(qb.w, bf16hi(kk.w), s3);
              u0 = fmaf(qb.x, bf16lo(k2.z), u0);
              u1 = fmaf(qb.y, bf16hi(k2.z), u1);
              u2 = fmaf(qb.z, bf16lo(k2.w), u2);
              u3 = fmaf(qb.w, bf16hi(k2.w), u3);
            }
            sdot2 = (u0 + u1) + (u2 + u3);
          } else {
  #pragma unroll
            for (int jj = 0; jj < 8; jj++) {
              const int jq = (jj + t) & 7;
              const uint4 kk = *reinterpret_cast<const uint4 *>(kr + 8 * jq);
              const float4 qa = *reinterpret_cast<const float4 *>(qh + 8 * jq);
              const float4 qb = *reinterpret_cast<const float4 *>(qh + 8 * jq + 4);
              s0 = fmaf(qa.x, bf16lo(kk.x), s0);
              s1 = fmaf(qa.y, bf16hi(kk.x), s1);
              s2 = fmaf(qa.z, bf16lo(kk.y), s2);
              s3 = fmaf(qa.w, bf16hi(kk.y), s3);
              s0 = fmaf(qb.x, bf16lo(kk.z), s0);
              s1 = fmaf(qb.y, bf16hi(kk.z), s1);
              s2 = fmaf(qb.z, bf16lo(kk.w), s2);
              s3 = fmaf(qb.w, bf16hi(kk.w), s3);
            }
          }
          sdot = (s0 + s1) + (s2 + s3);
        }
        sdot += __shfl_xor_sync(0xffffffffu, sdot, 16);
        sdot2 += __shfl_xor_sync(0xffffffffu, sdot2, 16);
        const float sc = (t < ntok) ? sdot * a.scale : -INFINITY;
        const float sc2 = (t < ntok2) ? sdot2 * a.scale : -INFINITY;
        float mx = fmaxf(sc, sc2);
  #pragma unroll
        for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float m_new = fmaxf(m_w, mx);
        const float pr = (t < ntok) ? expf(sc - m_new) : 0.f;
        const float pr2 = (t < ntok2) ? expf(sc2 - m_new) : 0.f;
        const float corr = (m_w == -INFINITY) ? 0.f : expf(m_w - m_new);
        l_w = l_w * corr + (pr + pr2);   // this lane's token shares; summed over the lanes after the loop
        m_w = m_new;
  #pragma unroll
        for (int e = 0; e < 4; e++) {
          acc4[e] *= corr;
          acc4b[e] *= corr;
        }
        // slots past the sequence end hold whatever the pool has there: skip them
        if (ntok == PAGE && ntok2 == PAGE) {
  #pragma unroll
          for (int tt = 0; tt < PAGE; tt++) {
            const float p_t = __shfl_sync(0xffffffffu, pr, tt);
            const float p2_t = __shfl_sync(0xffffffffu, pr2, tt);
            const uint2 vv = *reinterpret_cast<const uint2 *>(vb + tt * HD + 4 * lane);
            const uint2 v2 = *reinterpret_cast<const uint2 *>(vb2 + tt * HD + 4 * lane);
            acc4[0] = fmaf(p_t, bf16lo(vv.x), acc4[0]);
            acc4[1] = fmaf(p_t, bf16hi(vv.x), acc4[1]);
            acc4[2] = fmaf(p_t, bf16lo(vv.y), acc4[2]);
            acc4[3] = fmaf(p_t, bf16hi(vv.y), acc4[3]);
            acc4b[0] = fmaf(p2_t, bf16lo(v2.x), acc4b[0]);
            acc4b[1] = fmaf(p2_t, bf16hi(v2.x), acc4b[1]);
            acc4b[2] = fmaf(p2_t, bf16lo(v2.y), acc4b[2]);
            acc4b[3] = fmaf(p2_t, bf16hi(v2.y), acc4b[3]);
          }
        } else if (ntok == PAGE && ntok2 == 0) {
  #pragma unroll
          for (int tt = 0; tt < PAGE; tt++) {
            const float p_t = __shfl_sync(0xffffffffu, pr, tt);
            const uint2 vv = *reinterpret_cast<const uint2 *>(vb + tt * HD + 4 * lane);
            acc4[0] = fmaf(p_t, bf16lo(vv.x), acc4[0]);
            acc4[1] = fmaf(p_t, bf16hi(vv.x), acc4[1]);
            acc4[2] = fmaf(p_t, bf16lo(vv.y), acc4[2]);
            acc4[3] = fmaf(p_t, bf16hi(vv.y), acc4[3]);
          }
        } else {
          for (int tt = 0; tt < PAGE; tt++) {
            const float p_t = __shfl_sync(0xffffffffu, pr, tt);
            const float p2_t = __shfl_sync(0xffffffffu, pr2, tt);
            if (tt < ntok) {
              const uint2 vv = *reinterpret_cast<const uint2 *>(vb + tt * HD + 4 * lane);
              acc4[0] = fmaf(p_t, bf16lo(vv.x), acc4[0]);
              acc4[1] = fmaf(p_t, bf16hi(vv.x), acc4[1]);
              acc4[2] = fmaf(p_t, bf16lo(vv.y), acc4[2]);
              acc4[3] = fmaf(p_t, bf16hi(vv.y), acc4[3]);
            }
            if (tt < ntok2) {
              const uint2 v2 = *reinterpret_cast<const uint2 *>(vb2 + tt * HD + 4 * lane);
              acc4b[0] = fmaf(p2_t, bf16lo(v2.x), acc4b[0]);
              acc4b[1] = fmaf(p2_t, bf16hi(v2.x), acc4b[1]);
              acc4b[2] = fmaf(p2_t, bf16lo(v2.y), acc4b[2]);
              acc4b[3] = fmaf(p2_t, bf16hi(v2.y), acc4b[3]);
            }
          }
        }
        // both warps of the pair are done with the buffers: the head-0 warp
        // refills each with its stream position + NB
        bar_sync_n(1 + pw, 64);
        if (h == 0 && lane == 0) {
          const int tgt = i + NB, tgt2 = i2 + NB;   // item-relative; >= n: the next item's page tgt - n
          const bool r1 = tgt < n || tgt - n < nx_n;
          const bool r2 = two && (tgt2 < n || tgt2 - n < nx_n);
          if (r1 || r2) fence_proxy_async_smem();
          if (r1) attn_issue_pg(a, refill_page, tgt < n ? g : nx.g, ctr + NB, kc, smem_base);
          if (r2) attn_issue_pg(a, refill_page2, tgt2 < n ? g : nx.g, ctr2 + NB, kc, smem_base);
          if (r1 || r2) atomicMax(&kc.att_issued, (r2 ? ctr2 : ctr) + NB + 1u);
        }
      }
    } else {
      for (int i = pw; i < n; i += NWARPS / 2) {
        const unsigned ctr = kc.page_ctr + i;
        const int buf = ctr % NB;
        // every lane observes the phase flip, which makes the bulk-copied bytes
        // visible to it; the pair agrees on the outcome (named barrier 1 + pw),
        // so a timeout ends both warps' loops at the same page
        const bool landed = mbar_wait(kc.bars + buf, (ctr / NB) & 1u, WAIT_LIMIT_CYCLES);
        if (!bar_and_n(1 + pw, 64, landed)) {
          if (lane == 0 && !landed) raise_err(kc, ERR_MBAR_TIMEOUT, i);
          break;
        }
        uint16_t *kb = att_buf(smem_base, buf);
        uint16_t *vb = kb + PAGE * HD;
        const int pg = p_begin + i;
        const int ntok = min(PAGE, L - pg * PAGE);
        if (pg == npages - 1 && owns_new) {
          // the newest token comes from shared memory, not from the copy (both
          // warps of the page write the same bytes)
          const int slot = pos % PAGE;
          *reinterpret_cast<uint2 *>(kb + slot * HD + 4 * lane) = *reinterpret_cast<const uint2 *>(sm->knew + 4 * lane);
          *reinterpret_cast<uint2 *>(vb + slot * HD + 4 * lane) = *reinterpret_cast<const uint2 *>(sm->vnew + 4 * lane);
          __syncwarp();
        }
        // the page that will reuse this buffer: its index is loaded now, so
        // the refill at the end of the page does not wait for it
        int refill_page = -1;
        if (h == 0 && lane == 0) {
          const int tgt = i + NB;
          if (tgt < n) refill_page = __ldg(pt + p_begin + tgt);
          else if (tgt - n < nx_n) refill_page = __ldg(a.page_table + (size_t)nx.b * a.pt_stride + nx.p_begin + (tgt - n));
        }
        // score of token t: lanes t and t + 16 each take half of the 128 dims
        // in 16-byte groups, walking them from a token-dependent start so each
        // 8-lane phase of a 16-byte read hits 8 distinct bank groups; four
        // partial sums
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        const float *qh = sm->q[h] + half * 64;
        const uint16_t *kr = kb + t * HD + half * 64;
  #pragma unroll
        for (int jj = 0; jj < 8; jj++) {
          const int jq = (jj + t) & 7;
          const uint4 kk = *reinterpret_cast<const uint4 *>(kr + 8 * jq);
          const float4 qa = *reinterpret_cast<const float4 *>(qh + 8 * jq);
          const float4 qb = *reinterpret_cast<const float4 *>(qh + 8 * jq + 4);
          s0 = fmaf(qa.x, bf16lo(kk.x), s0);
          s1 = fmaf(qa.y, bf16hi(kk.x), s1);
          s2 = fmaf(qa.z, bf16lo(kk.y), s2);
          s3 = fmaf(qa.w, bf16hi(kk.y), s3);
          s0 = fmaf(qb.x, bf16lo(kk.z), s0);
          s1 = fmaf(qb.y, bf16hi(kk.z), s1);
          s2 = fmaf(qb.z, bf16lo(kk.w), s2);
          s3 = fmaf(qb.w, bf16hi(kk.w), s3);
        }
        float sdot = (s0 + s1) + (s2 + s3);
        sdot += __shfl_xor_sync(0xffffffffu, sdot, 16);
        const float sc = (t < ntok) ? sdot * a.scale : -INFINITY;
        float mx = sc;
  #pragma unroll
        for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float m_new = fmaxf(m_w, mx);
        const float pr = (t < ntok) ? expf(sc - m_new) : 0.f;
        const float corr = (m_w == -INFINITY) ? 0.f : expf(m_w - m_new);
        l_w = l_w * corr + pr;   // this lane's token share; summed over the lanes after the loop
        m_w = m_new;
  #pragma unroll
        for (int e = 0; e < 4; e++) acc4[e] *= corr;
        // slots past the sequence end hold whatever the pool has there: skip them
        if (ntok == PAGE) {
  #pragma unroll
          for (int tt = 0; tt < PAGE; tt++) {
            const float p_t = __shfl_sync(0xffffffffu, pr, tt);
            const uint2 vv = *reinterpret_cast<const uint2 *>(vb + tt * HD + 4 * lane);
            acc4[0] = fmaf(p_t, bf16lo(vv.x), acc4[0]);
            acc4[1] = fmaf(p_t, bf16hi(vv.x), acc4[1]);
            acc4[2] = fmaf(p_t, bf16lo(vv.y), acc4[2]);
            acc4[3] = fmaf(p_t, bf16hi(vv.y), acc4[3]);
          }
        } else {
          for (int tt = 0; tt < ntok; tt++) {
            const float p_t = __shfl_sync(0xffffffffu, pr, tt);
            const uint2 vv = *reinterpret_cast<const uint2 *>(vb + tt * HD + 4 * lane);
            acc4[0] = fmaf(p_t, bf16lo(vv.x), acc4[0]);
            acc4[1] = fmaf(p_t, bf16hi(vv.x), acc4[1]);
            acc4[2] = fmaf(p_t, bf16lo(vv.y), acc4[2]);
            acc4[3] = fmaf(p_t, bf16hi(vv.y), acc4[3]);
          }
        }
        // both warps of the pair are done with the buffer: the head-0 warp
        // refills it with stream position ctr + NB
        bar_sync_n(1 + pw, 64);
        const int tgt = i + NB;   // item-relative; >= n: the next item's page tgt - n
        if (h == 0 && lane == 0 && (tgt < n || tgt - n < nx_n)) {
          fence_proxy_async_smem();
          attn_issue_pg(a, refill_page, tgt < n ? g : nx.g, ctr + NB, kc, smem_base);
          atomicMax(&kc.att_issued, ctr + NB + 1u);
        }
      }
    }
#pragma unroll
    for (int e = 0; e < 4; e++) acc4[e] += acc4b[e];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) l_w += __shfl_xor_sync(0xffffffffu, l_w, o);
    // per-warp states -> per-head totals, in warp order
    float *s_acc = reinterpret_cast<float *>(smem + ATT_COMB_OFF);   // [NWARPS][HD]
    float *s_ml = s_acc + NWARPS * HD;                                // [NWARPS][2]
    *reinterpret_cast<float4 *>(s_acc + warp * HD + 4 * lane) = make_float4(acc4[0], acc4[1], acc4[2], acc4[3]);
    if (lane == 0) { s_ml[2 * warp] = m_w; s_ml[2 * warp + 1] = l_w; }
    if (__syncthreads_or(kc.local_err)) return;   // copies still in flight are drained on the way out
    if (tid == 0) kc.page_ctr += n;
    const int hh = tid >> 7, d = tid & 127;
    float Mh = -INFINITY;
#pragma unroll
    for (int q = 0; q < NWARPS / 2; q++) Mh = fmaxf(Mh, s_ml[2 * (2 * q + hh)]);
    float Lh = 0.f, acc = 0.f;
#pragma unroll
    for (int q = 0; q < NWARPS / 2; q++) {
      const int w = 2 * q + hh;
      const float mw = s_ml[2 * w];
      const float e = (mw == -INFINITY) ? 0.f : expf(mw - Mh);
      Lh += s_ml[2 * w + 1] * e;
      acc += s_acc[w * HD + d] * e;
    }
    ckpt(kc, 2);

    // ---- output / split combine ----
    const int head = 2 * g + hh;
    if (nsp == 1) {
      __stcg(a.out + (size_t)b * a.ld_out + head * HD + d, acc * (1.0f / Lh));
    } else {
      float *wsi = a.ws + ((((size_t)b * a.n_kv + g) * a.max_splits + sp) * 2 + hh) * (HD + 2);
      __stcg(wsi + d, acc);
      if (d == 0) { __stcg(wsi + HD, Mh); __stcg(wsi + HD + 1, Lh); }
      __threadfence();
      __syncthreads();
      if (tid == 0) sm->flag = (atomicAdd(a.sem + (size_t)b * a.n_kv + g, 1u) == (unsigned)(nsp - 1));
      __syncthreads();
      if (sm->flag) {
        __threadfence();
        const float *w0 = a.ws + ((((size_t)b * a.n_kv + g) * a.max_splits) * 2 + hh) * (HD + 2);
        float M = -INFINITY;
        for (int s2 = 0; s2 < nsp; s2++) M = fmaxf(M, __ldcg(w0 + (size_t)s2 * 2 * (HD + 2) + HD));
        float Ls = 0.f, O = 0.f;
        for (int s2 = 0; s2 < nsp; s2++) {
          const float *wsp = w0 + (size_t)s2 * 2 * (HD + 2);
          const float e = expf(__ldcg(wsp + HD) - M);
          Ls += __ldcg(wsp + HD + 1) * e;
          O += __ldcg(wsp + d) * e;
        }
        __stcg(a.out + (size_t)b * a.ld_out + head * HD + d, O * (1.0f / Ls));
        if (tid == 0) a.sem[(size_t)b * a.n_kv + g] = 0u;
      }
    }
    __syncthreads();
    item = next;
  }
  // every CTA took exactly one item past the end: the counter now stands at
  // the next dynamic stage's base
  if (a.dyn && threadIdx.x == 0) kc.att_base += (unsigned)n_items + gridDim.x;
}

// ATT_ATTEND (a prefill's attention): program slot b is one prompt token at
// position pos_ptr[b] of one sequence (slot b's page-table row holds that
// sequence's pages); it attends to positions 0 .. pos.  Positions before the
// prompt come from the bf16 pages, prompt positions from the f32 prompt
// buffer (a.pkv), as in the reference's prefill, which attends to its
// prompt's unrounded K/V (qwen_tts_talker.c:904-914, qwen_causal_attention at
// qwen_tts_kernels.c:3454).  One item per (slot, KV head), CTA + k * grid.
// Tiles of 16 positions go to the warp pairs in turn (pair pw: tiles pw,
// pw + 4, ...); the pair stages a tile's K and V in f32 in shared memory
// (two page buffers of its own), then each warp of the pair runs the online
// softmax of one query head over it, as the decode loop does per page; the
// per-warp states combine in warp order.  The result does not depend on the
// CTA that ran the item.
__device__ __noinline__ void attn_prefill_stage(const AttnArgs &a, int B, char *smem_base, KCtx &kc) {
  char *smem = smem_base + SM_X_OFF;
  AttnSmem *sm = reinterpret_cast<AttnSmem *>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  if (!a.pkv || !a.pos_ptr || a.nbuf < NWARPS) {
    if (tid == 0) raise_err(kc, ERR_BAD_STAGE, 3000 + a.nbuf);
    return;
  }
  const PromptKV P = *a.pkv;
  const int h = warp & 1, pw = warp >> 1;
  const int t = lane & 15, half = lane >> 4;
  float *kt = reinterpret_cast<float *>(att_buf(smem_base, 2 * pw));       // [PAGE][HD]
  float *vt = reinterpret_cast<float *>(att_buf(smem_base, 2 * pw + 1));   // [PAGE][HD]
  float *s_acc = reinterpret_cast<float *>(smem + ATT_COMB_OFF);            // [NWARPS][HD]
  float *s_ml = s_acc + NWARPS * HD;                                         // [NWARPS][2]
  const int n_items = B * a.n_kv;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int b = item / a.n_kv, g = item - b * a.n_kv;
    const int pos = __ldcg(a.pos_ptr + b);
    if (pos < 0 || pos >= a.rope_len || pos >= a.pt_stride * PAGE || pos < P.p0 || pos - P.p0 >= P.cap) {
      if (tid == 0) raise_err(kc, ERR_BAD_POS, pos);
      return;
    }
    const int *pt = a.page_table + (size_t)b * a.pt_stride;
    if (warp < 2) {
      float v[4];
      attn_row(a, b, g, warp, pos, lane, v);
#pragma unroll
      for (int i = 0; i < 4; i++) sm->q[warp][lane + 32 * i] = v[i];
    }
    __syncthreads();
    const int n = pos / PAGE + 1;
    const float *kf = P.k + ((size_t)a.layer * a.n_kv + g) * P.cap * HD;
    const float *vf = P.v + ((size_t)a.layer * a.n_kv + g) * P.cap * HD;
    float m_w = -INFINITY, l_w = 0.f, acc4[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = pw; i < n; i += NWARPS / 2) {
      // stage tile i: warp h of the pair takes rows h, h + 2, ..., lane the
      // 4 dims 4 lane .. 4 lane + 3; rows past pos are zeros
      float4 rk[PAGE / 2], rv[PAGE / 2];
      int page = 0;
      if (i * PAGE < P.p0) {
        page = __ldg(pt + i);
        if (page < 0 || page >= a.n_pages) {
          if (lane == 0) raise_err(kc, ERR_BAD_PAGE, page);
          page = 0;
        }
      }
#pragma unroll
      for (int k = 0; k < PAGE / 2; k++) {
        const int r = 2 * k + h, j = i * PAGE + r;
        rk[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        rv[k] = rk[k];
        if (j <= pos) {
          if (j >= P.p0) {
            const size_t off = (size_t)(j - P.p0) * HD + 4 * lane;
            rk[k] = __ldcg(reinterpret_cast<const float4 *>(kf + off));
            rv[k] = __ldcg(reinterpret_cast<const float4 *>(vf + off));
          } else {
            const size_t off = (((size_t)page * a.n_kv + g) * PAGE + r) * HD + 4 * lane;
            const uint2 kb = __ldcg(reinterpret_cast<const uint2 *>(a.kpool + off));
            const uint2 vb = __ldcg(reinterpret_cast<const uint2 *>(a.vpool + off));
            rk[k] = make_float4(bf16lo(kb.x), bf16hi(kb.x), bf16lo(kb.y), bf16hi(kb.y));
            rv[k] = make_float4(bf16lo(vb.x), bf16hi(vb.x), bf16lo(vb.y), bf16hi(vb.y));
          }
        }
      }
      bar_sync_n(1 + pw, 64);   // the pair is done with the previous tile
#pragma unroll
      for (int k = 0; k < PAGE / 2; k++) {
        const int r = 2 * k + h;
        *reinterpret_cast<float4 *>(kt + r * HD + 4 * lane) = rk[k];
        *reinterpret_cast<float4 *>(vt + r * HD + 4 * lane) = rv[k];
      }
      bar_sync_n(1 + pw, 64);
      // score of token t: lanes t and t + 16 each take half of the dims, in
      // 16-byte groups from a token-dependent start (distinct banks per
      // 8-lane phase)
      const float *qh = sm->q[h] + half * 64;
      const float *kr = kt + t * HD + half * 64;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int jj = 0; jj < 16; jj++) {
        const int jq = (jj + t) & 15;
        const float4 kk = *reinterpret_cast<const float4 *>(kr + 4 * jq);
        const float4 qq = *reinterpret_cast<const float4 *>(qh + 4 * jq);
        s0 = fmaf(qq.x, kk.x, s0);
        s1 = fmaf(qq.y, kk.y, s1);
        s2 = fmaf(qq.z, kk.z, s2);
        s3 = fmaf(qq.w, kk.w, s3);
      }
      float sdot = (s0 + s1) + (s2 + s3);
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 16);
      const bool live = i * PAGE + t <= pos;
      const float sc = live ? sdot * a.scale : -INFINITY;
      float mx = sc;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_w, mx);   // finite: position i * PAGE <= pos
      const float pr = live ? expf(sc - m_new) : 0.f;
      const float corr = (m_w == -INFINITY) ? 0.f : expf(m_w - m_new);
      l_w = l_w * corr + pr;
      m_w = m_new;
#pragma unroll
      for (int e = 0; e < 4; e++) acc4[e] *= corr;
#pragma unroll
      for (int tt = 0; tt < PAGE; tt++) {
        const float p_t = __shfl_sync(0xffffffffu, pr, tt);
        const float4 vv = *reinterpret_cast<const float4 *>(vt + tt * HD + 4 * lane);
        acc4[0] = fmaf(p_t, vv.x, acc4[0]);
        acc4[1] = fmaf(p_t, vv.y, acc4[1]);
        acc4[2] = fmaf(p_t, vv.z, acc4[2]);
        acc4[3] = fmaf(p_t, vv.w, acc4[3]);
      }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) l_w += __shfl_xor_sync(0xffffffffu, l_w, o);
    *reinterpret_cast<float4 *>(s_acc + warp * HD + 4 * lane) = make_float4(acc4[0], acc4[1], acc4[2], acc4[3]);
    if (lane == 0) { s_ml[2 * warp] = m_w; s_ml[2 * warp + 1] = l_w; }
    if (__syncthreads_or(kc.local_err)) return;
    const int hh = tid >> 7, d = tid & 127;
    float Mh = -INFINITY;
#pragma unroll
    for (int q = 0; q < NWARPS / 2; q++) Mh = fmaxf(Mh, s_ml[2 * (2 * q + hh)]);
    float Lh = 0.f, acc = 0.f;
#pragma unroll
    for (int q = 0; q < NWARPS / 2; q++) {
      const int w = 2 * q + hh;
      const float mw = s_ml[2 * w];
      const float e = (mw == -INFINITY) ? 0.f : expf(mw - Mh);
      Lh += s_ml[2 * w + 1] * e;
      acc += s_acc[w * HD + d] * e;
    }
    __stcg(a.out + (size_t)b * a.ld_out + (2 * g + hh) * HD + d, acc * (1.0f / Lh));
    __syncthreads();   // q, the tiles and the states are rewritten by the next item
  }
}

// ============================================================ misc stages ==
__device__ __noinline__ void embed_stage(const EmbedArgs &e, int B, KCtx &kc) {
  const int total = B * e.dim;
  for (int idx = blockIdx.x * NTHREADS + threadIdx.x; idx < total; idx += gridDim.x * NTHREADS) {
    const int b = idx / e.dim, i = idx - b * e.dim;
    // all codes first, then all table rows: independent loads in flight together
    int c[16];
#pragma unroll
    for (int t = 0; t < 16; t++) c[t] = (t < e.ntab) ? __ldcg(e.code[t] + (size_t)b * e.code_stride[t]) : 0;
    const float f = e.fsrc ? __ldcg(e.fsrc + (size_t)b * e.fsrc_ld + i) : 0.f;
    const float ad = e.add ? __ldg(e.add + i) : 0.f;
    uint16_t r[16];
#pragma unroll
    for (int t = 0; t < 16; t++) {
      if (t < e.ntab) {
        if (c[t] < 0 || c[t] >= e.tab_rows[t]) { if (i == 0) raise_err(kc, ERR_BAD_CODE, c[t]); c[t] = 0; }
        r[t] = __ldg(e.tab[t] + (size_t)c[t] * e.tab_ld[t] + i);
      }
    }
    float v = f;
#pragma unroll
    for (int t = 0; t < 16; t++)
      if (t < e.ntab) v += __uint_as_float(((uint32_t)r[t]) << 16);
    if (e.add) v += ad;
    __stcg(e.dst + (size_t)b * e.ld_dst + i, v);
  }
}

__device__ __noinline__ void norm_stage(const NormArgs &n, int B) {
  __shared__ float s_red[NWARPS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int MAXV = 8;   // dim <= 2048
  for (int b = blockIdx.x; b < B; b += gridDim.x) {
    const float *xb = n.x + (size_t)b * n.ldx;
    float xv[MAXV], wv[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV; j++) {
      const int i = threadIdx.x + j * NTHREADS;
      xv[j] = (i < n.dim) ? __ldcg(xb + i) : 0.f;
      wv[j] = (i < n.dim) ? __ldg(n.w + i) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < MAXV; j++) ss += xv[j] * xv[j];
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NWARPS; w++) tot += s_red[w];
    const float inv = 1.0f / sqrtf(tot / (float)n.dim + n.eps);
#pragma unroll
    for (int j = 0; j < MAXV; j++) {
      const int i = threadIdx.x + j * NTHREADS;
      if (i < n.dim) __stcg(n.y + (size_t)b * n.ldy + i, (xv[j] * inv) * wv[j]);
    }
    __syncthreads();
  }
}

// Second half of the grid barrier, thread 0 polling.  While the other CTAs
// finish, the hook issues the independent loads of the coming stage -- the
// older K/V pages of an attention stage, the weights of a GEMV stage -- one
// step per poll, so a barrier that completes stops the hook within one step.
// The CTA whose arrival completed the barrier skips both (an error raised
// elsewhere reaches it at a later barrier, or the host at the end).  Advances
// the stage counters.
QTB_DEV bool grid_wait(KCtx &kc, char *smem) {
  __shared__ int s_ok;
  if (kc.cl) {
    // the hook once (the cluster barrier has no poll loop), then the barrier
    if (threadIdx.x < 32) {
      const unsigned nxt = kc.seq + 1;
      if (nxt < kc.n_total) {
        const int slot = (int)(nxt % NDESC);
        const bool landed = __all_sync(0xffffffffu, mbar_test(kc.dbars + slot, (nxt / NDESC) & 1u));
        if (landed && kc.dring[slot].kind == ST_ATTN && kc.dring[slot].a.mode == ATT_DECODE)
          attn_prefetch(kc.dring[slot].a, kc.dring[slot].B, kc, smem);
        __syncwarp();
        if (threadIdx.x == 0 && landed) {
          const Stage *nx = kc.dring + slot;
          if (nx->kind == ST_GEMV && nx->g.v2) prefetch_gemv_operands(nx->g, kc.pring[slot]);
        }
        __syncwarp();
      }
    }
    __syncwarp();
    cluster_wait();
    const int tag = kc.cl_err;
    const bool ok = !(tag != 0 && tag <= (int)kc.epoch + 1);
    __syncthreads();   // every thread has read the tag and the hook's state
    if (threadIdx.x == 0) {
      kc.epoch++;
      kc.seq++;
      kc.stage = (kc.stage + 1 == kc.n_stages) ? 0 : kc.stage + 1;
    }
    __syncthreads();
    return ok;
  }
  if (threadIdx.x < 32) {   // warp 0: lane 0 polls, the warp runs the hook
    const int lane = threadIdx.x;
    __syncwarp();            // kc.last, written by lane 0 in grid_arrive
    int ok = kc.local_err ? 0 : 1;   // a CTA that raised an error leaves after arriving
    if (ok && !kc.last) {
      const unsigned target = (kc.epoch + 1u) * gridDim.x;
      const unsigned nxt = kc.seq + 1;
      // hook steps: 0 the coming attention stage's first pages, 1 weights two
      // stages ahead, 2 the coming GEMV stage's small operands; before a GEMV
      // stage the weights go first (a short wait may allow one step only)
      int phase = (nxt < kc.n_total) ? 0 : 3;
      if (phase == 0) {   // warp-uniform: every lane tests the descriptor's barrier
        const int s0 = (int)(nxt % NDESC);
        if (__all_sync(0xffffffffu, mbar_test(kc.dbars + s0, (nxt / NDESC) & 1u)) && kc.dring[s0].kind == ST_GEMV)
          phase = 1;
      }
      const long long t0 = clock64();
      unsigned spins = 0;
      while (true) {
        uint2 w = make_uint2(0u, 0u);
        if (lane == 0) w = ld_acquire_gpu_v2(&kc.ctl->bar_count);   // {count, err}
        w.x = __shfl_sync(0xffffffffu, w.x, 0);
        w.y = __shfl_sync(0xffffffffu, w.y, 0);
        if (w.y != 0u) { ok = 0; break; }
        if ((int)(w.x - target) >= 0) break;
        const int slot = (int)(nxt % NDESC);
        if (phase == 0) {
          // every lane tests the descriptor's barrier itself (that makes the
          // bulk-copied descriptor visible to it)
          const bool landed = __all_sync(0xffffffffu, mbar_test(kc.dbars + slot, (nxt / NDESC) & 1u));
          if (landed && kc.dring[slot].kind == ST_ATTN && kc.dring[slot].a.mode == ATT_DECODE)
            attn_prefetch(kc.dring[slot].a, kc.dring[slot].B, kc, smem);
          __syncwarp();
          phase = 1;
        } else if (phase == 1) {
          // this stage's and the next one's weights: two stages of lead time
          stream(kc, smem, nxt, nxt + 2);
          phase = 2;
        } else if (phase == 2) {
          // the coming GEMV stage's small operands into L2
          if (lane == 0 && mbar_test(kc.dbars + slot, (nxt / NDESC) & 1u)) {
            const Stage *nx = kc.dring + slot;
            if (nx->kind == ST_GEMV && nx->g.v2) prefetch_gemv_operands(nx->g, kc.pring[slot]);
          }
          __syncwarp();
          phase = 3;
        }
        const int late = __shfl_sync(0xffffffffu, (++spins & 31u) == 0 && clock64() - t0 > WAIT_LIMIT_CYCLES, 0);
        if (late) {
          if (lane == 0) raise_err(kc, ERR_BARRIER_TIMEOUT, (int)kc.epoch);
          ok = 0;
          break;
        }
      }
    }
    if (lane == 0) {
      s_ok = ok;
      kc.epoch++;
      kc.seq++;
      kc.stage = (kc.stage + 1 == kc.n_stages) ? 0 : kc.stage + 1;
    }
  }
  __syncthreads();
  return s_ok != 0;
}

// The codec-head sampler alone (qtb_codec_sample_host): block b, one warp,
// samples row b of the logits in g.
__global__ void __launch_bounds__(32) sample_kernel(const GenState *g, int *out) {
  const int r = sample_codec(g, blockIdx.x);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

// ====================================================== persistent kernel ==
__global__ void __launch_bounds__(NTHREADS, 1)
decode_kernel(const Stage *__restrict__ prog, const V2Plan *__restrict__ plan, int n_stages, int n_iters, Ctl *ctl,
              long long *trace, int cl) {
  extern __shared__ __align__(128) char smem[];
  __shared__ __align__(8) uint64_t bars[ATT_NBUF_MAX];
  __shared__ __align__(8) uint64_t wbars[NWSLOT];
  __shared__ __align__(8) uint64_t dbars[NDESC];
  __shared__ Stage dring[NDESC];   // stage descriptors, NDESC - 1 stages ahead
  __shared__ V2Plan pring[NDESC];  // this CTA's plan entries for them ([stage][CTA] in `plan`)
  __shared__ __align__(8) uint64_t pbar;
  __shared__ __align__(8) uint64_t tcbars[2 * TC_NSLOT + 2];   // weight slot full / empty, accumulators
  __shared__ __align__(8) uint64_t clbars[2 * NWARPS];          // single-cluster GEMV: per-warp weight slots
  __shared__ uint32_t tmem_base;
  __shared__ KCtx kc;
  if (threadIdx.x == 0) {
    kc.epoch = 0;
    kc.page_ctr = 0;
    kc.wfill = 0;
    kc.att_issued = 0;
    kc.att_nbuf = ATT_NBUF;
    kc.att_base = 0;   // ctl->att_work is zeroed before the launch
    kc.att_first = -1;
    kc.att_tot = 0;
    kc.local_err = 0;
    kc.wbars = wbars;
    kc.pol_first = policy_evict_first();
    kc.pol_last = policy_evict_last();
    kc.bars = bars;
    kc.ctl = ctl;
    kc.stage = 0;
    kc.trace2 = trace ? trace + (size_t)n_iters * n_stages + 1 : nullptr;
    kc.trace_cta = trace ? ctl->trace_cta : 0;
    kc.gtrace = trace ? reinterpret_cast<unsigned long long *>(trace + (size_t)n_iters * n_stages + 1 +
                                                               (size_t)n_stages * NCKPT)
                      : nullptr;
    kc.seq = 0;
    kc.n_total = (unsigned)n_stages * (unsigned)n_iters;
    kc.n_stages = n_stages;
    kc.dring = dring;
    kc.pring = pring;
    kc.pbar = &pbar;
    kc.pair_ctr = 0;
    kc.dbars = dbars;
    kc.w_issued = 0;
    kc.w_free = 0;
    kc.pf_seq = 0;
    kc.pf_f = 0;
    kc.tcfull = tcbars;
    kc.tcempty = tcbars + TC_NSLOT;
    kc.tcacc = tcbars + 2 * TC_NSLOT;
    kc.tc_issued = 0;
    kc.tc_done = 0;
    kc.tc_committed = 0;
    kc.tc_waited = 0;
    kc.ibar_target = 0;
    kc.cl = cl;
    kc.clbars = clbars;
    for (int w = 0; w < NWARPS; w++) {
      kc.cl_q[w] = 0u;
      kc.cl_iss[w] = 0u;
      kc.cl_pre[w] = ~0u;
    }
    kc.cl_err = 0;
  }
  // the tensor-memory accumulator of the tcgen05 GEMV stages, held for the
  // whole launch (one CTA per SM: the allocation never waits)
  if (threadIdx.x < 32) tmem_alloc(&tmem_base, TC_TMEM_COLS);
  auto issue_desc = [&](unsigned k) {   // thread 0: descriptor (+ plan entry) of stage k into its slot
    const int slot = (int)(k % NDESC);
    const unsigned si = k % (unsigned)n_stages;
    mbar_arrive_expect_tx(dbars + slot, sizeof(Stage) + (plan ? sizeof(V2Plan) : 0));
    bulk_g2s(dring + slot, prog + si, sizeof(Stage), dbars + slot);
    if (plan) bulk_g2s(pring + slot, plan + (size_t)si * gridDim.x + blockIdx.x, sizeof(V2Plan), dbars + slot);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < ATT_NBUF_MAX; i++) mbar_init(bars + i, 1);
    for (int i = 0; i < NWSLOT; i++) mbar_init(wbars + i, 1);
    for (int i = 0; i < NDESC; i++) mbar_init(dbars + i, 1);
    for (int i = 0; i < 2 * TC_NSLOT + 2; i++) mbar_init(tcbars + i, 1);
    mbar_init(&pbar, 1);
    for (int i = 0; i < 2 * NWARPS; i++) mbar_init(clbars + i, 1);
    fence_mbar_init();
    for (unsigned k = 0; k < NDESC - 1 && k < kc.n_total; k++) issue_desc(k);
    kc.t_start = clock64();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) kc.tmem = tmem_base;
  __syncthreads();
  if (cl) {   // every CTA's error word is initialised before any CTA can write to it
    cluster_arrive();
    cluster_wait();
  }
  if (trace && blockIdx.x == 0 && threadIdx.x == 0) trace[(size_t)n_iters * n_stages] = clock64();
  for (int it = 0; it < n_iters; it++) {
    for (int si = 0; si < n_stages; si++) {
      const unsigned seq = kc.seq;
      const int slot = (int)(seq % NDESC);
      if (!mbar_wait(dbars + slot, (seq / NDESC) & 1u, WAIT_LIMIT_CYCLES)) raise_err(kc, ERR_MBAR_TIMEOUT, -1);
      if (threadIdx.x == 0 && seq + NDESC - 1 < kc.n_total) {
        // the slot of stage seq - 1 is free: every thread left that stage
        fence_proxy_async_smem();
        issue_desc(seq + NDESC - 1);
      }
      const Stage *st = dring + slot;
      const int B = st->B;
      switch (st->kind) {
        case ST_GEMV: gemv_stage(st->g, B, smem, kc); break;
        case ST_ATTN:
          if (st->a.mode == ATT_ATTEND) attn_prefill_stage(st->a, B, smem, kc);
          else attn_stage(st->a, B, smem, kc);
          break;
        case ST_EMBED: embed_stage(st->e, B, kc); break;
        case ST_NORM: norm_stage(st->n, B); break;
        case ST_POS_INC:
          // done = 1: the slot sampled EOS in this frame, whose talker step
          // did run (its position advances past it, as the reference's does),
          // and it stops: done = 2 keeps its position and frame count
          if (blockIdx.x == 0)
            for (int b = threadIdx.x; b < B; b += NTHREADS) {
              const GenState *gs = st->p.gen;
              const int d = (gs && gs->enabled) ? __ldcg(gs->done + b) : 0;
              if (d >= 2) continue;
              st->p.pos[b] += 1;
              if (gs && gs->enabled) {
                gs->frame[b] += 1;
                if (d == 1) gs->done[b] = 2;
              }
            }
          break;
        default:
          if (threadIdx.x == 0 && blockIdx.x == 0) raise_err(kc, ERR_BAD_STAGE, st->kind);
          break;
      }
      ckpt(kc, 6);
      grid_arrive(kc);
      ckpt(kc, 7);
      if (kc.gtrace && threadIdx.x == 0) {
        // [stage][cta] = global arrival time; [n_stages + stage][cta] = this CTA's
        // busy cycles since it left the previous barrier (same-SM clock) | smid << 48
        unsigned smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        kc.gtrace[(size_t)si * gridDim.x + blockIdx.x] = globaltimer();
        kc.gtrace[(size_t)(n_stages + si) * gridDim.x + blockIdx.x] =
            (unsigned long long)(clock64() - kc.t_start) | ((unsigned long long)smid << 48);
      }
      if (!grid_wait(kc, smem)) {   // (advances kc.seq and kc.stage)
        if (threadIdx.x == 0) drain(kc, seq);
        tc_fence_before();
        __syncthreads();
        if (threadIdx.x < 32) tmem_dealloc(kc.tmem, TC_TMEM_COLS);
        return;
      }
      if (threadIdx.x == 0) kc.t_start = clock64();
      // optional stage trace: CTA 0's clock when every CTA has finished stage si
      if (trace && blockIdx.x == 0 && threadIdx.x == 0) trace[(size_t)it * n_stages + si] = clock64();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) tmem_dealloc(kc.tmem, TC_TMEM_COLS);
}

}  // namespace qtb
