// Persistent weight-streaming decode step of libqwenb200: the whole token
// (embed, 24 layers, tied head, argmax) in ONE cooperative launch with one
// CTA per SM.
//
// Weight streamer.  Every CTA owns a ring of NSLOT shared-memory slots (16 KB
// of weight rows + the rows' fp32 scales).  A static per-CTA schedule lists
// the weight chunks (contiguous rows of one matrix) the CTA consumes during
// the token, in consumption order.  Each slot is refilled with cp.async.bulk
// (L2 evict-first, completion on the slot's mbarrier) by whichever of the
// eight warps finishes reading it last (a per-slot shared-memory counter), so
// the HBM stream runs ahead of the compute by the ring's depth wherever the
// compute is waiting -- the decoupled weight-stationary streaming the
// reference's HBM engine is built around (docs/hbm_bandwidth.md), on 148 SMs.
// Warps never synchronise with each other per chunk.
//
// No grid barriers.  Activations crossing CTAs are 64-bit words {fp32 value,
// 32-bit tag} written with relaxed gpu-scope stores; tag = step_seq*128 +
// phase + 1 is unique per (token, phase).  A consumer polls exactly the words
// it needs (all of a thread's loads issued before any is checked) until every
// tag matches.  The split-KV attention merge and the head argmax use
// last-arriver counters.  Every wait is bounded by %globaltimer; on expiry the
// CTA records ERR_WAIT, raises a global abort flag that every other wait also
// watches, drains its in-flight bulk copies and returns.
//
// Phase program per layer l (p = 5l + sub): IN (projections of the normed
// residual), MIX (DeltaNet delta rule, or split-KV attention), OUT (out/o
// projection + residual), GATEUP (silu(gate)*up), DOWN (down projection +
// residual); phase 120 is the tied head, on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, accumulators in tensor memory) over a copy of the
// embedding re-tiled at load time into the canonical K-major layout.
//
// A phase's chunks are a precomputed index range of the CTA's list (counted
// loops; the schedule stores where every phase starts).  Arithmetic (and its rounding order)
// is that of decode.cu, so both engines agree bit for bit; the contract is
// golden/model.py:243-267.
#include <algorithm>
#include <cstdio>
#include <string>
#include <vector>

#include "common.cuh"
#include "persist.cuh"

namespace qb {
// The device code has internal linkage: persist_tp.cu compiles this file again.
namespace {

constexpr int NCW = 16;                 // warps per CTA
constexpr int PT = NCW * 32;            // threads per CTA
constexpr int NTHREADS = PT;
constexpr int SLOTW = 16384;            // weight bytes per ring slot
constexpr int SLOT = SLOTW;             // slot stride
constexpr int NSLOT = 11;               // ring depth
constexpr int MAXCH = 448;              // chunk-list capacity per CTA
constexpr int NPHASE = PERSIST_NPHASE;  // 121
constexpr int PH_HEAD = NLAYER * 5;
constexpr int MAXP = (KMAX / 2 + PT - 1) / PT;  // tagged pairs per thread in a full-vector wait (4)
constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s bound on any wait



// ---- shared memory layout (dynamic, offsets from the aligned base)
constexpr int OFF_RING = 0;
constexpr int DIG_BYTES = 3 * KMAX;                       // the digit image (see dig_off)
constexpr int OFF_DIG = OFF_RING + NSLOT * SLOT;
constexpr int OFF_XF = OFF_DIG + DIG_BYTES;               // float [KMAX]
constexpr int OFF_HS = OFF_XF + 4 * KMAX;                 // float [HID]
constexpr int MAXPAN = NSLOT;                             // panels of one phase on one CTA (at most)
constexpr int OFF_PART = OFF_HS + 4 * HID;                // int [MAXPAN][4][PANEL]: exact digit sums
constexpr int OFF_PSC = OFF_PART + 4 * MAXPAN * 4 * PANEL;   // float [MAXPAN][PANEL]: the panels' row scales
constexpr int OFF_LAY = OFF_PSC + 4 * MAXPAN * PANEL;     // LayerW [NLAYER]
constexpr int OFF_CH = OFF_LAY + ((int)sizeof(LayerW) * NLAYER + 15) / 16 * 16;  // Chunk [MAXCH]
constexpr int OFF_BAR = OFF_CH + 8 * MAXCH;               // u64 mbarriers, see bar_* below
constexpr int NBAR = 3 * NSLOT + 5;                       // full, (spare), mma per slot; acc_full[2], acc_empty[2], fin
constexpr int OFF_MISC = OFF_BAR + 8 * NBAR;              // small scalars
// tensor-core phases: the x digits as the B operand (16 rows x HID, canonical
// K-major layout: rows 0-2 the digit planes, 3-15 zero; 8-row groups BT_SBO
// bytes apart), over the digit planes and xf, which the head does not use
constexpr int BT_SBO = (HID / 16) * 128;
constexpr int OFF_BT = OFF_DIG;
static_assert(OFF_BT % 128 == 0 && OFF_BT + 2 * BT_SBO <= OFF_HS, "head B tile");
constexpr int MISC_BYTES = 1152;
constexpr int SMEM_BYTES = OFF_MISC + MISC_BYTES;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert(OFF_DIG % 16 == 0 && OFF_XF % 16 == 0 && OFF_HS % 16 == 0 && SLOT % 16 == 0, "alignment");
static_assert(OFF_BAR % 8 == 0 && OFF_MISC % 8 == 0, "alignment");
static_assert(MAXP * 2 * PT >= KMAX, "pair split");

struct Misc {
  unsigned tmem;           // tensor memory base (accumulators), written by tcgen05.alloc
  unsigned pad_[3];
  float red[48];
  int pend_min;
  int ntile;               // tensor-core tiles this CTA has issued so far in the step
  unsigned mpar;           // refiller: per-slot parity of the next MMA-completion phase
  int mma_any;             // the issuer has issued at least one MMA this launch
  unsigned hs_tag;         // tag of the residual stream held in hs (0: none)
  double scale;
  int ndig;
  int abort;
  int tok;
  int last;
  int slot_last[NSLOT];    // last chunk issued into the slot (-1: none)
  unsigned short pf[NPHASE + 1];  // this CTA's chunk range of each phase (phase_first)
  int pos, T, conv_base, act_int8, want_logits, seq, step;
  unsigned long long wbest[NCW];
  float inv_h[LH];
  float gate_g, gate_beta;
  float abv[2];            // DeltaNet head CTA: the head's in_proj_b, in_proj_a outputs
  float ssw[NCW];          // per-warp sums of squares of a normed GEMV input
  int pcnt[NSLOT];         // GEMV phase: tasks finished per panel (the last one finishes the panel)
  int rfq[NCW][2];         // per warp: ring slots to refill at the next phase (first | count << 16)
  float xinv;              // 1/rms of the current normed GEMV input (W8A32 path)
  unsigned amax[2];        // bits of max|v| of the GEMV input of phases p with p & 1 = index
};
static_assert(sizeof(Misc) <= MISC_BYTES, "misc");
static_assert(OFF_MISC % 16 == 0, "tcgen05.alloc destination alignment");

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Named barrier 1 over all 512 threads.  The non-.aligned forms: a warp may
// reach them with its lanes not yet reconverged (lane-0 work just before).
__device__ __forceinline__ void consumer_sync() {
  __syncwarp();
  asm volatile("barrier.sync 1, 512;" ::: "memory");
}
__device__ __forceinline__ int consumer_or(int v) {
  int r;
  __syncwarp();
  asm volatile("{ .reg .pred p, q; setp.ne.s32 p, %1, 0; barrier.red.or.pred q, 1, 512, p; selp.s32 %0, 1, 0, q; }"
               : "=r"(r) : "r"(v) : "memory");
  return r;
}
__device__ __forceinline__ int consumer_and(int v) {
  int r;
  __syncwarp();
  asm volatile("{ .reg .pred p, q; setp.ne.s32 p, %1, 0; barrier.red.and.pred q, 1, 512, p; selp.s32 %0, 1, 0, q; }"
               : "=r"(r) : "r"(v) : "memory");
  return r;
}
__device__ __forceinline__ void ld_tv2(const unsigned long long* p, unsigned long long& a,
                                       unsigned long long& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0,%1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tv(const unsigned long long* p) {
  unsigned long long a;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
  return a;
}
__device__ __forceinline__ void st_tv(unsigned long long* p, float v, unsigned tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" :: "l"(p), "l"(w) : "memory");
}
// Tagged words crossing GPUs (the TP exchange buffers, written over NVLink):
// system scope.
__device__ __forceinline__ unsigned long long ld_tv_sys(const unsigned long long* p) {
  unsigned long long a;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
  return a;
}
__device__ __forceinline__ void st_tv_sys(unsigned long long* p, float v, unsigned tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" :: "l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ int ld_flag(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool tag_ok(unsigned long long w, unsigned tag) {
  return (unsigned)(w >> 32) == tag;
}
__device__ __forceinline__ float tv_val(unsigned long long w) { return __uint_as_float((unsigned)w); }
__device__ __forceinline__ void mbar_init(unsigned bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned bar, unsigned parity) {
  unsigned ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Non-blocking probe of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(unsigned bar, unsigned parity) {
  unsigned ok;
  asm volatile("{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Shared-memory counter with acquire / release semantics at CTA scope.
__device__ __forceinline__ int atom_add_acq_rel_cta(int* p, int v) {
  int r;
  asm volatile("atom.acq_rel.cta.shared::cta.add.s32 %0, [%1], %2;"
               : "=r"(r) : "r"((unsigned)__cvta_generic_to_shared(p)), "r"(v) : "memory");
  return r;
}
__device__ __forceinline__ void mbar_arrive(unsigned bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void bulk_g2s(unsigned dst, const void* src, unsigned bytes, unsigned bar,
                                         unsigned long long pol) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}
__device__ __forceinline__ void mbar_expect(unsigned bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- kernel context
struct PCtx {
  const PersistArgs* A;
  unsigned char* sm;
  Misc* ms;
  LayerW* lay;
  const Chunk* ch;
  int nch;          // chunks of this CTA
  unsigned long long pol;
};

__device__ __forceinline__ unsigned full_bar(const PCtx& c, int slot) { return smem_u32(c.sm + OFF_BAR + 8 * slot); }

// tcgen05 completion of the MMAs that read slot s (head phase)
__device__ __forceinline__ unsigned mma_bar(const PCtx& c, int slot) {
  return smem_u32(c.sm + OFF_BAR + 8 * (2 * NSLOT + slot));
}
// head accumulator buffer b: MMAs done (acc_full) / epilogue done reading it (acc_empty)
__device__ __forceinline__ unsigned accf_bar(const PCtx& c, int b) { return smem_u32(c.sm + OFF_BAR + 8 * (3 * NSLOT + b)); }
__device__ __forceinline__ unsigned acce_bar(const PCtx& c, int b) { return smem_u32(c.sm + OFF_BAR + 8 * (3 * NSLOT + 2 + b)); }
__device__ __forceinline__ unsigned fin_bar(const PCtx& c) { return smem_u32(c.sm + OFF_BAR + 8 * (3 * NSLOT + 4)); }

// ---------------------------------------------------------------- tcgen05 (5th-gen tensor cores)

// Shared-memory matrix descriptor, canonical K-major layout without swizzle:
// start address, leading byte offset (between the two 16-byte core-matrix
// columns of one MMA's K = 32), stride byte offset (between 8-row groups),
// descriptor version 1.
__device__ __forceinline__ unsigned long long umma_desc(unsigned addr, unsigned lbo, unsigned sbo) {
  return (unsigned long long)((addr >> 4) & 0x3fffu) | (unsigned long long)((lbo >> 4) & 0x3fffu) << 16 |
         (unsigned long long)((sbo >> 4) & 0x3fffu) << 32 | 1ull << 46;
}
// Instruction descriptor of kind::i8: s32 accumulators, signed int8 A and B,
// both K-major, N columns, M rows.
__host__ __device__ constexpr unsigned umma_idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((unsigned)(N >> 3) << 17) | ((unsigned)(M >> 4) << 24);
}
// D[tmem] (+)= A[M x 32] * B[N x 32]^T, one int8 K-step; issued by one thread.
__device__ __forceinline__ void umma_i8(unsigned tmem, unsigned long long a, unsigned long long b,
                                        unsigned idesc, unsigned accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
               :: "r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive (once) on an mbarrier when every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(unsigned bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ unsigned tag_of(const PCtx& c, int phase) {
  return (unsigned)c.ms->seq * 128u + (unsigned)phase + 1u;
}

__device__ __forceinline__ void trace_mark(const PCtx& c, int p, int k) {
  if (c.A->trace && threadIdx.x == 0)
    c.A->trace[((size_t)blockIdx.x * NPHASE + p) * TRACE_STAMPS + k] = gtime();
}
// The same stamp from any thread, keeping the latest (the record is zeroed
// before a traced step).
__device__ __forceinline__ void trace_latest(const PCtx& c, int p, int k) {
  if (c.A->trace) atomicMax(c.A->trace + ((size_t)blockIdx.x * NPHASE + p) * TRACE_STAMPS + k, gtime());
}
// per-warp stamps of the first GEMV CTA (after the per-phase block): [phase][warp][TRACE_WARP_STAMPS]
// SM clock cycles (clock64), finer than the global timer.  Compiled in only
// with QB_WARP_TRACE defined (every call site costs instructions on the hot
// path, traced or not); otherwise that part of the record stays zero.
__device__ __forceinline__ void trace_warp(const PCtx& c, int p, int k) {
#ifdef QB_WARP_TRACE
  if (c.A->trace && (int)blockIdx.x == c.A->dn_h1 - c.A->dn_h0 && (threadIdx.x & 31) == 0)
    c.A->trace[(size_t)gridDim.x * NPHASE * TRACE_STAMPS +
               ((size_t)p * NCW + (threadIdx.x >> 5)) * TRACE_WARP_STAMPS + k] = clock64();
#else
  (void)c; (void)p; (void)k;
#endif
}

// Record a device error (first one wins: code, site, value and, for ERR_WAIT,
// the CTA in err[1..3]) and stop every CTA.  One copy in the kernel (not
// inlined, plain arguments): the error paths of every site share it.
__device__ __noinline__ void record_error(int* err, int* abort_flag, Misc* ms, int code, int site, int value) {
  if (atomicCAS(err, 0, code) == 0) {
    err[1] = site;
    err[2] = value;
    if (code == ERR_WAIT) err[3] = (int)blockIdx.x;
  }
  atomicExch(abort_flag, 1);
  *(volatile int*)&ms->abort = 1;
}
// A device-side bounds check failed (the access itself is skipped by the caller).
__device__ __forceinline__ void check_fail(const PCtx& c, int site, int value) {
  record_error(c.A->err, c.A->abort_flag, c.ms, ERR_CHECK, site, value);
}
// A bounded wait ran out (or the schedule is unusable).
__device__ __forceinline__ void raise_abort(const PCtx& c, int site = 0, int value = 0) {
  record_error(c.A->err, c.A->abort_flag, c.ms, ERR_WAIT, site, value);
}
__device__ __forceinline__ bool aborted(const PCtx& c) {
  return *(volatile int*)&c.ms->abort || ld_flag(c.A->abort_flag);
}

// K window [k0, k1) of GEMV phase `sub` packed as k0 | k1 << 16: the whole
// input (IN, GATEUP), or the rank's input columns of a row-parallel OUT / DOWN.
__host__ __device__ __forceinline__ unsigned kwin_of(int sub, unsigned kw_out, unsigned kw_down) {
  return sub == 2 ? kw_out : (sub == 4 ? kw_down : (unsigned)HID << 16);
}
__device__ __forceinline__ unsigned kwin(const PersistArgs& A, int sub) {
  return kwin_of(sub, (unsigned)A.ok0 | (unsigned)A.ok1 << 16, (unsigned)A.dk0 | (unsigned)A.dk1 << 16);
}
// The same in a kernel instance: TP = false compiles the whole-input windows in.
template <bool TP>
__device__ __forceinline__ unsigned kwin_t(const PersistArgs& A, int sub) {
  if constexpr (TP) return kwin(A, sub);
  else return kwin_of(sub, (unsigned)VDIM << 16, (unsigned)FFN << 16);
}

// Source and size of chunk k: one K-slice of a layer panel (slice n covers
// K [k0 + 1024 n, min(k0 + 1024 (n + 1), k1)) of the phase's window), or one
// K-slab of a head tile.  src = null for a chunk outside its matrix.
__device__ __forceinline__ void chunk_src(const LayerW* lay, const int8_t* head_tiles, const Chunk& k,
                                          unsigned kw_out, unsigned kw_down, const char*& src,
                                          unsigned& bytes) {
  const int p = k.phase;
  const int row0 = (int)k.row0, n = k.nrows;
  src = nullptr;
  bytes = 0;
  if (k.seg & CHUNK_MMA) {   // row scales are read by the epilogue
    if (p != PH_HEAD || row0 >= HEAD_TILES || n >= HEAD_NSLAB) return;
    src = (const char*)head_tiles + ((size_t)row0 * HEAD_NSLAB + n) * SLOTW;
    bytes = SLOTW;
    return;
  }
  if (p >= PH_HEAD) return;
  const LayerW& L = lay[p / 5];
  const int sub = p % 5;
  if (k.seg & CHUNK_PANEL) {   // row scales are read at the end of the phase
    const int8_t* base = nullptr;
    int np = 0;
    size_t pbytes = 0;
    if (sub == 0) { base = L.pin; np = (L.linear ? CONVD + VDIM : QPROJ + 2 * KVPROJ) / PANEL; pbytes = (size_t)PANEL * HID; }
    else if (sub == 2) { base = L.pout; np = HID / PANEL; pbytes = (size_t)PANEL * VDIM; }
    else if (sub == 3) { base = L.pgu; np = FFN / PAIR_ROWS; pbytes = (size_t)PANEL * HID; }
    else if (sub == 4) { base = L.pdown; np = HID / PANEL; pbytes = (size_t)PANEL * FFN; }
    const unsigned kw = kwin_of(sub, kw_out, kw_down);
    const int k0 = (int)(kw & 0xffffu) + n * PANEL_KB, k1 = (int)(kw >> 16);
    if (!base || row0 >= np || k0 >= k1 || (size_t)k1 * PANEL > pbytes) return;
    src = (const char*)base + (size_t)row0 * pbytes + (size_t)k0 * PANEL;
    const int kl = k1 - k0 < PANEL_KB ? k1 - k0 : PANEL_KB;
    bytes = (unsigned)(kl * PANEL);
    return;
  }
}

// Issue the bulk copy of chunk i into its slot (one lane).  One copy in the
// kernel (not inlined, plain arguments): every refill site calls it.
__device__ __noinline__ void issue_chunk_core(const Chunk* ch, const LayerW* lay, const int8_t* head_tiles,
                                              unsigned kw_out, unsigned kw_down, unsigned char* sm,
                                              unsigned long long pol, int* err, int* abort_flag, int i) {
  const int slot = i % NSLOT;
  const Chunk k = ch[i];
  const char* src;
  unsigned bytes;
  chunk_src(lay, head_tiles, k, kw_out, kw_down, src, bytes);
  if (!src) {   // a chunk outside its matrix: ERR_CHECK site 5, every CTA stops
    record_error(err, abort_flag, (Misc*)(sm + OFF_MISC), ERR_CHECK, 5, (int)k.row0);
    return;
  }
  const unsigned bar = smem_u32(sm + OFF_BAR + 8 * slot);   // full_bar
  mbar_expect(bar, bytes);
  bulk_g2s(smem_u32(sm + OFF_RING + slot * SLOT), src, bytes, bar, pol);
}
__device__ __forceinline__ void issue_chunk(const PCtx& c, int i) {
  issue_chunk_core(c.ch, c.lay, c.A->head_tiles, kwin(*c.A, 2), kwin(*c.A, 4), c.sm, c.pol, c.A->err,
                   c.A->abort_flag, i);
}

// One thread: bounded wait for phase `parity` of an mbarrier.  false on abort
// or time-out (which raises the abort).
__device__ bool wait_bar1(const PCtx& c, unsigned bar, unsigned parity, int site, int value) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtime();
  int it = 0;
  while (!mbar_try(bar, parity)) {
    if (((++it) & 63) == 0) {
      if (aborted(c)) return false;
      if (gtime() - t0 > WAIT_NS) { raise_abort(c, site, value); return false; }
    }
  }
  return true;
}

// Whole warp: bounded wait on an mbarrier phase (every lane polls: when the
// phase has completed, as it usually has, that is one probe per lane).  Same
// result in every lane.
__device__ __forceinline__ bool wait_bar_warp(PCtx& c, unsigned bar, unsigned parity, int site, int value) {
  int good = 1;
  if (!mbar_test(bar, parity)) {
    const unsigned long long t0 = gtime();
    int it = 0;
    while (!mbar_try(bar, parity)) {
      if (((++it) & 63) == 0) {
        if (aborted(c)) { good = 0; break; }
        if (gtime() - t0 > WAIT_NS) { raise_abort(c, site, value); good = 0; break; }
      }
    }
  }
  return __all_sync(0xffffffffu, good) != 0;
}
// Consumer warp: wait for chunk i's bytes.  Same result in every lane.
__device__ __forceinline__ bool wait_full(PCtx& c, int i) {
  return wait_bar_warp(c, full_bar(c, i % NSLOT), (unsigned)((i / NSLOT) & 1), 11, i);
}

// Poll tagged words src[0..n) (n even, n <= KMAX) until all carry `tag`; values
// into dst (smem).  Each thread issues all its pending loads before checking
// any.  Collective over the consumer threads.  false on abort.  One copy in
// the kernel (not inlined): every phase's input wait runs the same
// instructions.
//
// With amax (a shared word, zero on entry; may be null) the wait also folds
// max|v| of the values into it (red.shared.max on the bits of a non-negative
// float orders like the floats), v = the value, or value * (1 + g) with the
// thread's norm gains g (gain, for n = 2 * PT: one pair per thread).  The
// barrier that ends the wait publishes it.  With ssw (may be null), every
// warp writes the sum of v^2 over its values (the raw values) to ssw[warp]
// after the wait; the caller's next CTA barrier publishes them.
__device__ __noinline__ bool wait_tagged_words(Misc* ms, int* err, int* abort_flag,
                                               const unsigned long long* src, int n, unsigned tag,
                                               float* dst, unsigned* amax, bool gain, float2 g2,
                                               float* ssw) {
  const unsigned long long t0 = gtime();
  float ss = 0.0f;
  const int npair = n >> 1;
  unsigned pend = 0;
#pragma unroll
  for (int j = 0; j < MAXP; ++j)
    if ((int)threadIdx.x + PT * j < npair) pend |= 1u << j;
  float vmax = 0.0f;
  bool folded = false;
  int it = 0;
  for (;;) {
    unsigned long long a[MAXP], b[MAXP];
#pragma unroll
    for (int j = 0; j < MAXP; ++j)
      if (pend >> j & 1) ld_tv2(src + 2 * (threadIdx.x + PT * j), a[j], b[j]);
#pragma unroll
    for (int j = 0; j < MAXP; ++j) {
      if ((pend >> j & 1) && tag_ok(a[j], tag) && tag_ok(b[j], tag)) {
        const int q = threadIdx.x + PT * j;
        const float v0 = tv_val(a[j]), v1 = tv_val(b[j]);
        dst[2 * q] = v0;
        dst[2 * q + 1] = v1;
        if (gain) vmax = fmaxf(vmax, fmaxf(fabsf(__fmul_rn(v0, __fadd_rn(1.0f, g2.x))),
                                           fabsf(__fmul_rn(v1, __fadd_rn(1.0f, g2.y)))));
        else vmax = fmaxf(vmax, fmaxf(fabsf(v0), fabsf(v1)));
        ss = fmaf(v1, v1, fmaf(v0, v0, ss));
        pend &= ~(1u << j);
      }
    }
    if (amax) {
      // lanes whose values all arrived fold their max once: one shared atomic per warp
      const bool nw = pend == 0 && !folded;
      const unsigned wm = __reduce_max_sync(0xffffffffu, nw ? __float_as_uint(vmax) : 0u);
      if (nw) folded = true;
      if ((threadIdx.x & 31) == 0 && wm)
        asm volatile("red.shared.max.u32 [%0], %1;" :: "r"(smem_u32(amax)), "r"(wm) : "memory");
    }
    if (consumer_and(pend == 0)) {
      if (ssw) {   // published by the caller's next barrier
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) ssw[threadIdx.x >> 5] = ss;
      }
      return true;
    }
    if (((++it) & 15) == 0) {
      int bad = 0;
      if (threadIdx.x == 0) {
        if (*(volatile int*)&ms->abort || ld_flag(abort_flag)) {
          bad = 1;
        } else if (gtime() - t0 > WAIT_NS) {
          record_error(err, abort_flag, ms, ERR_WAIT, 12, (int)(tag & 127u));
          bad = 1;
        }
      }
      if (!consumer_and(!bad)) return false;
    }
  }
}
__device__ __forceinline__ bool wait_tagged(PCtx& c, const unsigned long long* src, int n, unsigned tag,
                                            float* dst) {
  return wait_tagged_words(c.ms, c.A->err, c.A->abort_flag, src, n, tag, dst, nullptr, false,
                           make_float2(0.0f, 0.0f), nullptr);
}

// One run of tagged words a GEMV phase waits for: np pairs from src into dst
// (shared memory), all carrying `tag`.
struct WSeg {
  const unsigned long long* src;
  float* dst;
  int np;
  unsigned tag;
};
constexpr int MAXW = 5;   // pairs per thread over a GEMV phase's segments (DeltaNet OUT: o, z, residual)

// The input wait of a GEMV phase: the words of up to three segments polled
// together (all of a thread's pending loads issued before any is checked)
// until every one carries its segment's tag; values into the segments' dst.
// Pair q = tid + PT j of the concatenated segments.  Segment 0 is the
// projection input: with amax, max|v| over its values folds into *amax (v =
// value * (1 + g) with the thread's norm gains g2 when `gain`: a normed input
// is segment 0 alone, HID values, thread t = pair t), and with ssw each warp
// writes the sum of value^2 over its segment-0 values to ssw[warp] (the
// caller's next barrier publishes it).  Collective; false on abort.  Inlined
// into the GEMV phase (one call site), so the task registers loaded before
// it are not saved across a call.
__device__ __forceinline__ bool wait_inputs(Misc* ms, int* err, int* abort_flag, const WSeg& s0, const WSeg& s1,
                                            const WSeg& s2, unsigned* amax, bool gain, float2 g2, float* ssw) {
  const unsigned long long t0 = gtime();
  const int n01 = s0.np + s1.np, ntot = n01 + s2.np;
  unsigned pend = 0;
#pragma unroll
  for (int j = 0; j < MAXW; ++j)
    if ((int)threadIdx.x + PT * j < ntot) pend |= 1u << j;
  float vmax = 0.0f, ss = 0.0f;
  bool folded = false;
  int it = 0;
  for (;;) {
    unsigned long long a[MAXW], b[MAXW];
#pragma unroll
    for (int j = 0; j < MAXW; ++j) {
      if (!(pend >> j & 1)) continue;
      const int q = (int)threadIdx.x + PT * j;
      const unsigned long long* sp = q < s0.np ? s0.src + 2 * q
                                   : (q < n01 ? s1.src + 2 * (q - s0.np) : s2.src + 2 * (q - n01));
      ld_tv2(sp, a[j], b[j]);
    }
#pragma unroll
    for (int j = 0; j < MAXW; ++j) {
      if (!(pend >> j & 1)) continue;
      const int q = (int)threadIdx.x + PT * j;
      const int sg = q < s0.np ? 0 : (q < n01 ? 1 : 2);
      const unsigned tag = sg == 0 ? s0.tag : (sg == 1 ? s1.tag : s2.tag);
      if (!tag_ok(a[j], tag) || !tag_ok(b[j], tag)) continue;
      float* d = sg == 0 ? s0.dst + 2 * q : (sg == 1 ? s1.dst + 2 * (q - s0.np) : s2.dst + 2 * (q - n01));
      const float v0 = tv_val(a[j]), v1 = tv_val(b[j]);
      d[0] = v0;
      d[1] = v1;
      if (sg == 0) {
        if (gain) vmax = fmaxf(vmax, fmaxf(fabsf(__fmul_rn(v0, __fadd_rn(1.0f, g2.x))),
                                           fabsf(__fmul_rn(v1, __fadd_rn(1.0f, g2.y)))));
        else vmax = fmaxf(vmax, fmaxf(fabsf(v0), fabsf(v1)));
        ss = fmaf(v1, v1, fmaf(v0, v0, ss));
      }
      pend &= ~(1u << j);
    }
    if (amax) {
      // lanes whose values all arrived fold their max once: one shared atomic per warp
      const bool nw = pend == 0 && !folded;
      const unsigned wm = __reduce_max_sync(0xffffffffu, nw ? __float_as_uint(vmax) : 0u);
      if (nw) folded = true;
      if ((threadIdx.x & 31) == 0 && wm)
        asm volatile("red.shared.max.u32 [%0], %1;" :: "r"(smem_u32(amax)), "r"(wm) : "memory");
    }
    if (consumer_and(pend == 0)) {
      if (ssw) {
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) ssw[threadIdx.x >> 5] = ss;
      }
      return true;
    }
    if (((++it) & 15) == 0) {
      int bad = 0;
      if (threadIdx.x == 0) {
        if (*(volatile int*)&ms->abort || ld_flag(abort_flag)) {
          bad = 1;
        } else if (gtime() - t0 > WAIT_NS) {
          record_error(err, abort_flag, ms, ERR_WAIT, 12, (int)(s0.tag & 127u));
          bad = 1;
        }
      }
      if (!consumer_and(!bad)) return false;
    }
  }
}

// ---------------------------------------------------------------- prologues

// The shared digit image of the GEMV input is kept in the B-fragment order of
// mma.m16n8k32: K-step s (positions 32s .. 32s+31) is 96 bytes, 12 lanes x 8
// bytes, lane 4d + u = digit d at positions 32s + 4u .. +3, then 32s + 16 + 4u
// .. +3.  Byte offset of the 4 positions k .. k+3 (k a multiple of 4) of digit d:
// 2^e as a float for -126 <= e <= 127.
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

__device__ __forceinline__ int dig_off(int d, int k) {
  return (k >> 5) * 96 + (d * 4 + ((k >> 2) & 3)) * 8 + ((k >> 4) & 1) * 4;
}

// W8A32 digit image of v = src[k0 .. k1) (a normed input: v = src * (1 + g),
// gains g from `gains`; may be null) into the CTA's image, as three UNSIGNED
// int8 digits: X = rint(v * 2^sh) with |X| <= 2^22 from the exact max|v|
// whose bits the input wait folded into amax, held as U = X + 2^22 in
// [0, 2^23].  v * 2^sh + 1.5 * 2^23 rounds once to an integer in [2^23, 2^24]
// whose float bits carry U in bytes 0-2 (U = 2^23 at the top end shows as
// byte 2 = 0x80): those bytes are the digits D0, D1, D2 (U = D0 + 256 D1 +
// 65536 D2), gathered with byte permutes.  The panel MMA multiplies them as
// unsigned against the signed weights and removes the 2^22 offset with the
// rows' weight sums (a column of ones).  Thread = groups of 4 positions
// (4 tid + 4 PT j); one 32-bit store per digit plane.  Returns 2^-sh (0: all
// zero).  Ends with a CTA barrier.
__device__ __forceinline__ float encode_u8(unsigned char* sm, const float* src, int k0, int k1, unsigned amax,
                                           const float* gains) {
  unsigned char* dg = sm + OFF_DIG;
  const int sh = 22 - ((int)((amax >> 23) & 0xffu) - 126);   // max in [2^(ex-1), 2^ex)
  const bool live = amax != 0u && sh <= 126;
  const float p2 = live ? pow2f(sh) : 0.0f;
  for (int g = (k0 >> 2) + threadIdx.x; g < (k1 >> 2); g += PT) {
    float4 x = *reinterpret_cast<const float4*>(src + 4 * g);
    if (gains) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(gains) + g);
      x.x = __fmul_rn(x.x, __fadd_rn(1.0f, w.x));
      x.y = __fmul_rn(x.y, __fadd_rn(1.0f, w.y));
      x.z = __fmul_rn(x.z, __fadd_rn(1.0f, w.z));
      x.w = __fmul_rn(x.w, __fadd_rn(1.0f, w.w));
    }
    const unsigned f0 = __float_as_uint(__fmaf_rn(x.x, p2, 12582912.0f));
    const unsigned f1 = __float_as_uint(__fmaf_rn(x.y, p2, 12582912.0f));
    const unsigned f2 = __float_as_uint(__fmaf_rn(x.z, p2, 12582912.0f));
    const unsigned f3 = __float_as_uint(__fmaf_rn(x.w, p2, 12582912.0f));
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      const unsigned sel = (unsigned)(d | (4 + d) << 4);
      *reinterpret_cast<unsigned*>(dg + dig_off(d, 4 * g)) =
          __byte_perm(__byte_perm(f0, f1, sel), __byte_perm(f2, f3, sel), 0x5410u);
    }
  }
  consumer_sync();
  return live ? pow2f(-sh) : 0.0f;
}

// Recombine the digit sums in fp32: (a2 * 65536 + a1 * 256 + a0) * (x_scale * s_w).
// Two fp32 roundings instead of the graph engine's single fp64 one (|rel| < 2e-7).
__device__ __forceinline__ float finish_f32(int a0, int a1, int a2, int ndig, float xs_sw) {
  float y = (float)a0;
  if (ndig == 3) y = fmaf((float)a2, 65536.0f, fmaf((float)a1, 256.0f, y));
  return y * xs_sw;
}


// Digit image of xf[0..K) (W8A32, three digits), or the golden _qa int8
// quantiser (ACT_INT8, one digit), into the fragment-ordered digit image.
// Same values as encode_x in common.cuh.
__device__ __noinline__ void encode_lin_core(unsigned char* sm, Misc* ms, int K, bool act_int8) {
  float* xf = (float*)(sm + OFF_XF);
  int8_t* dg = (int8_t*)(sm + OFF_DIG);
  float m = 0.0f;
  for (int i = threadIdx.x; i < K; i += PT) m = fmaxf(m, fabsf(xf[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) ms->red[threadIdx.x >> 5] = m;
  consumer_sync();
  float amax = 0.0f;
#pragma unroll
  for (int w = 0; w < NCW; ++w) amax = fmaxf(amax, ms->red[w]);
  // every thread handles 4 consecutive elements -> one 32-bit word per plane
  if (act_int8) {
    const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    for (int i4 = threadIdx.x; i4 < K / 4; i4 += PT) {
      unsigned w0 = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * i4 + e;
        int qi = 0;
        if (amax > 0.0f) {
          const float q = fminf(fmaxf(rintf(__fdiv_rn(xf[i], s)), -127.0f), 127.0f);
          xf[i] = __fmul_rn(q, s);
          qi = (int)q;
        }
        w0 |= ((unsigned)qi & 0xffu) << (8 * e);
      }
      *reinterpret_cast<unsigned*>(dg + dig_off(0, 4 * i4)) = w0;
    }
    if (threadIdx.x == 0) { ms->scale = (double)s; ms->ndig = 1; }
  } else {
    const int ex = amax > 0.0f ? (int)((__float_as_uint(amax) >> 23) & 0xff) - 126 : 0;
    const int sh = 22 - ex;               // amax in [2^(ex-1), 2^ex) for normal amax
    const bool fast = (__float_as_uint(amax) >> 23) != 0 && sh >= -126 && sh <= 127;
    const float p2 = fast ? pow2f(sh) : 0.0f;
    int exs = 0;
    if (!fast && amax > 0.0f) frexpf(amax, &exs);
    const int shs = fast ? sh : 22 - exs;
    for (int i4 = threadIdx.x; i4 < K / 4; i4 += PT) {
      unsigned w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v = xf[4 * i4 + e];
        int X = 0;
        if (amax > 0.0f) X = fast ? __float2int_rn(v * p2) : (int)rintf(ldexpf(v, shs));
        const int a0 = (X << 24) >> 24;
        const int X1 = (X - a0) >> 8;
        const int a1 = (X1 << 24) >> 24;
        const int a2 = (X1 - a1) >> 8;
        w0 |= ((unsigned)a0 & 0xffu) << (8 * e);
        w1 |= ((unsigned)a1 & 0xffu) << (8 * e);
        w2 |= ((unsigned)a2 & 0xffu) << (8 * e);
      }
      *reinterpret_cast<unsigned*>(dg + dig_off(0, 4 * i4)) = w0;
      *reinterpret_cast<unsigned*>(dg + dig_off(1, 4 * i4)) = w1;
      *reinterpret_cast<unsigned*>(dg + dig_off(2, 4 * i4)) = w2;
    }
    if (threadIdx.x == 0) { ms->scale = ldexp(1.0, -shs); ms->ndig = 3; }
  }
  consumer_sync();
}
__device__ __forceinline__ void encode_lin(PCtx& c, int K, bool act_int8) {
  encode_lin_core(c.sm, c.ms, K, act_int8);
}


// CTA-level encode of a normed HID input (every thread two elements, 2t and
// 2t+1): the sum of squares in numpy's pairwise order by warps 0-1 (the order
// of np.mean(x**2), golden/model.py:74), then 1/rms, x = h * inv * (1 + w), the
// digit image (the shift from an upper bound of max|x|) or, under ACT_INT8,
// the golden quantiser with the exact max|x| (golden/model.py:37-45).  Digits
// land in the fragment-ordered digit image (and x itself, fake-quantised under
// ACT_INT8, in xf), or (canon) in rows 0-2 (ACT_INT8: row 0) of the
// tensor-core B tile at OFF_BT with the other rows zeroed; returns inv and
// (ACT_INT8) s_x.  Two barriers (three under ACT_INT8).  One copy in the
// kernel (not inlined), shared by the IN, GATEUP and head phases.
__device__ __noinline__ float2 encode_normed(unsigned char* sm, Misc* ms, const float* hs, float2 g2,
                                             bool act_int8, bool canon, unsigned long long* tw) {
  int8_t* dg = (int8_t*)(sm + OFF_DIG);
  float inv_out = 0.0f, sx_out = 0.0f;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const float2 h2 = *reinterpret_cast<const float2*>(hs + 2 * t);
  const float w0 = __fadd_rn(1.0f, g2.x), w1 = __fadd_rn(1.0f, g2.y);
  if (wid < 2) {
    const int ch = lane + 32 * wid;          // chain: block ch / 8, accumulator ch % 8
    const float* a = hs + 128 * (ch >> 3) + (ch & 7);
    float acc = __fmul_rn(a[0], a[0]);
#pragma unroll
    for (int i = 1; i < 16; ++i) acc = __fadd_rn(acc, __fmul_rn(a[8 * i], a[8 * i]));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));   // (r0+r1), ...
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));   // ((r0+r1)+(r2+r3)), ...
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));   // block sums
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 8));   // (B0+B1), ...
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 16));  // ((B0+B1)+(B2+B3))
    if (lane == 0) ms->red[wid] = acc;
  }
  const float mb = warp_max(fmaxf(fabsf(h2.x * w0), fabsf(h2.y * w1)));
  if (lane == 0) ms->red[2 + wid] = mb;
  if (tw) tw[8] = clock64();
  consumer_sync();
  if (tw) tw[9] = clock64();
  const float tot = __fadd_rn(ms->red[0], ms->red[1]);
  // (tot / HID: HID is a power of two, so the product by 1/HID is the same
  // number; 1 / sqrt through the correctly rounded reciprocal, the same number
  // as the correctly rounded quotient)
  const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(tot, 1.0f / HID), EPS)));
  inv_out = inv;
  const float x0 = __fmul_rn(__fmul_rn(h2.x, inv), w0);
  const float x1 = __fmul_rn(__fmul_rn(h2.y, inv), w1);
  if (act_int8) {
    const float m = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
    if (lane == 0) ms->red[18 + wid] = m;
    consumer_sync();
    float amax = 0.0f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) amax = fmaxf(amax, ms->red[18 + w]);
    const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    int q0 = 0, q1 = 0;
    if (amax > 0.0f) {
      q0 = (int)fminf(fmaxf(rintf(__fdiv_rn(x0, s)), -127.0f), 127.0f);
      q1 = (int)fminf(fmaxf(rintf(__fdiv_rn(x1, s)), -127.0f), 127.0f);
    }
    const unsigned short qq = (unsigned short)(((unsigned)q0 & 0xffu) | (((unsigned)q1 & 0xffu) << 8));
    if (canon) {
      // B tile: row 0 = the int8 activations, rows 1-15 zero
      unsigned char* bt = sm + OFF_BT + ((2 * t) >> 4) * 128 + ((2 * t) & 15);
      *reinterpret_cast<unsigned short*>(bt) = qq;
#pragma unroll
      for (int d = 1; d < 8; ++d) *reinterpret_cast<unsigned short*>(bt + 16 * d) = 0;
#pragma unroll
      for (int d = 0; d < 8; ++d) *reinterpret_cast<unsigned short*>(bt + BT_SBO + 16 * d) = 0;
      fence_async_smem();
    } else {
      *reinterpret_cast<unsigned short*>(dg + dig_off(0, (2 * t) & ~3) + ((2 * t) & 2)) = qq;
      // x as the golden fake quantiser rebuilds it, for the fp32 rows
      *reinterpret_cast<float2*>(sm + OFF_XF + 8 * t) = make_float2(__fmul_rn((float)q0, s), __fmul_rn((float)q1, s));
    }
    if (t == 0) { ms->scale = (double)s; ms->ndig = 1; }
    sx_out = s;
  } else {
    float mbound = 0.0f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) mbound = fmaxf(mbound, ms->red[2 + w]);
    // max|x| <= inv * max|h (1 + w)| up to two roundings: the shift keeps |X| <= 2^22 + 1
    const float amax = mbound * inv;
    const int ex = amax > 0.0f ? (int)((__float_as_uint(amax) >> 23) & 0xff) - 126 : 0;
    int sh = 22 - ex;
    const bool fast = (__float_as_uint(amax) >> 23) != 0 && sh >= -126 && sh <= 127;
    if (!fast && amax > 0.0f) { int exs = 0; frexpf(amax, &exs); sh = 22 - exs; }
    int X[2] = {0, 0};
    if (amax > 0.0f) {
      if (fast) { const float p2 = pow2f(sh); X[0] = __float2int_rn(x0 * p2); X[1] = __float2int_rn(x1 * p2); }
      else { X[0] = (int)rintf(ldexpf(x0, sh)); X[1] = (int)rintf(ldexpf(x1, sh)); }
    }
    unsigned w_[3] = {0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int a0 = (X[e] << 24) >> 24;
      const int X1 = (X[e] - a0) >> 8;
      const int a1 = (X1 << 24) >> 24;
      const int a2 = (X1 - a1) >> 8;
      w_[0] |= ((unsigned)a0 & 0xffu) << (8 * e);
      w_[1] |= ((unsigned)a1 & 0xffu) << (8 * e);
      w_[2] |= ((unsigned)a2 & 0xffu) << (8 * e);
    }
    if (canon) {
      // elements 2t, 2t+1 sit in core-matrix column (2t)/16 of the 8 x HID tile
      unsigned char* bt = sm + OFF_BT + ((2 * t) >> 4) * 128 + ((2 * t) & 15);
#pragma unroll
      for (int d = 0; d < 3; ++d) *reinterpret_cast<unsigned short*>(bt + 16 * d) = (unsigned short)w_[d];
#pragma unroll
      for (int d = 3; d < 8; ++d) *reinterpret_cast<unsigned short*>(bt + 16 * d) = 0;
#pragma unroll
      for (int d = 0; d < 8; ++d) *reinterpret_cast<unsigned short*>(bt + BT_SBO + 16 * d) = 0;
      fence_async_smem();
    } else {
#pragma unroll
      for (int d = 0; d < 3; ++d)
        *reinterpret_cast<unsigned short*>(dg + dig_off(d, (2 * t) & ~3) + ((2 * t) & 2)) = (unsigned short)w_[d];
      *reinterpret_cast<float2*>(sm + OFF_XF + 8 * t) = make_float2(x0, x1);   // x itself, for the fp32 rows
    }
    if (t == 0) { ms->scale = ldexp(1.0, -sh); ms->ndig = 3; }
    sx_out = 0.0f;
  }
  if (tw) tw[10] = clock64();
  consumer_sync();
  return make_float2(inv_out, sx_out);
}
__device__ __forceinline__ void cta_encode_1024(PCtx& c, const float* hs, float2 g2, bool act_int8,
                                                float& inv_out, float& sx_out, bool canon = false,
                                                int tp = -1) {
  unsigned long long* tw = nullptr;
#ifdef QB_WARP_TRACE
  if (tp >= 0 && c.A->trace && (int)blockIdx.x == c.A->dn_h1 - c.A->dn_h0 && (threadIdx.x & 31) == 0)
    tw = c.A->trace + (size_t)gridDim.x * NPHASE * TRACE_STAMPS +
         ((size_t)tp * NCW + (threadIdx.x >> 5)) * TRACE_WARP_STAMPS;
#endif
  const float2 r = encode_normed(c.sm, c.ms, hs, g2, act_int8, canon, tw);
  inv_out = r.x;
  sx_out = r.y;
}

// W8A8 under tensor parallelism: the golden per-vector quantiser
// (golden/model.py:37-45) of the OUT / DOWN input, of which this rank holds the
// window [k0, k1) in xf.  The window's max|x| goes to every rank's exchange
// buffer; the max over all ranks' gives s_x = max / 127 as on one GPU, and the
// window is quantised with it into digit plane 0 (x itself fake-quantised in
// xf).  Collective; bounded wait; false on abort.
__device__ bool tp_encode_i8(PCtx& c, int p, int k0, int k1) {
  const PersistArgs& A = *c.A;
  Misc* ms = c.ms;
  float* xf = (float*)(c.sm + OFF_XF);
  int8_t* dg = (int8_t*)(c.sm + OFF_DIG);
  float m = 0.0f;
  for (int i = k0 + threadIdx.x; i < k1; i += PT) m = fmaxf(m, fabsf(xf[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) ms->red[threadIdx.x >> 5] = m;
  consumer_sync();
  int bad = 0;
  if (threadIdx.x == 0) {
    float lm = 0.0f;
    for (int w = 0; w < NCW; ++w) lm = fmaxf(lm, ms->red[w]);
    const unsigned tag = tag_of(c, p);
    const size_t slot = XB_AMAX + (size_t)(p % 5 == 4) * TP_MAX;
    for (int rr = 0; rr < A.tp_world; ++rr) st_tv_sys(A.xbuf[rr] + slot + A.tp_rank, lm, tag);
    const unsigned long long* xb = A.xbuf[A.tp_rank] + slot;
    const unsigned long long t0 = gtime();
    int it = 0;
    for (;;) {
      float g = 0.0f;
      bool all = true;
      for (int rr = 0; rr < A.tp_world && all; ++rr) {
        const unsigned long long w = ld_tv_sys(xb + rr);
        all = tag_ok(w, tag);
        g = fmaxf(g, tv_val(w));
      }
      if (all) { ms->red[NCW] = g; break; }
      if (((++it) & 63) == 0) {
        if (aborted(c)) { bad = 1; break; }
        if (gtime() - t0 > WAIT_NS) { raise_abort(c, 25, p); bad = 1; break; }
      }
    }
  }
  if (!consumer_and(!bad)) return false;
  const float amax = ms->red[NCW];
  const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  for (int i4 = (k0 >> 2) + threadIdx.x; i4 < (k1 >> 2); i4 += PT) {
    unsigned w0 = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * i4 + e;
      int qi = 0;
      if (amax > 0.0f) {
        const float q = fminf(fmaxf(rintf(__fdiv_rn(xf[i], s)), -127.0f), 127.0f);
        xf[i] = __fmul_rn(q, s);
        qi = (int)q;
      }
      w0 |= ((unsigned)qi & 0xffu) << (8 * e);
    }
    *reinterpret_cast<unsigned*>(dg + dig_off(0, 4 * i4)) = w0;
  }
  if (threadIdx.x == 0) { ms->scale = (double)s; ms->ndig = 1; }
  consumer_sync();
  return true;
}

// Tensor parallelism: this rank's packed (value, index) maximum of its vocab
// slice to every rank, then the maximum over all ranks' (one thread, bounded
// wait).  Packed maxima order by value, then by the lower index, so the
// result is the first index of the global maximum on every rank.
__device__ unsigned long long tp_argmax(PCtx& c, unsigned long long b) {
  const PersistArgs& A = *c.A;
  const unsigned tag = tag_of(c, PH_HEAD);
  const size_t off = XB_HEAD + 2 * (size_t)A.tp_rank;
  for (int rr = 0; rr < A.tp_world; ++rr) {
    st_tv_sys(A.xbuf[rr] + off, __uint_as_float((unsigned)(b >> 32)), tag);
    st_tv_sys(A.xbuf[rr] + off + 1, __uint_as_float((unsigned)b), tag);
  }
  const unsigned long long* xb = A.xbuf[A.tp_rank] + XB_HEAD;
  const unsigned long long t0 = gtime();
  int it = 0;
  for (;;) {
    unsigned long long g = 0ull;
    bool all = true;
    for (int rr = 0; rr < A.tp_world && all; ++rr) {
      const unsigned long long hi = ld_tv_sys(xb + 2 * rr), lo = ld_tv_sys(xb + 2 * rr + 1);
      all = tag_ok(hi, tag) && tag_ok(lo, tag);
      g = umax64(g, (unsigned long long)(unsigned)hi << 32 | (unsigned)lo);
    }
    if (all) return g;
    if (((++it) & 63) == 0) {
      if (aborted(c)) return b;
      if (gtime() - t0 > WAIT_NS) { raise_abort(c, 24, A.tp_rank); return b; }
    }
  }
}

// Block argmax of the head, then the last CTA reduces every block's maximum,
// records the step's argmax and advances the step scalars for the next launch.
template <bool TP>
__device__ void head_finish(PCtx& c, unsigned long long best) {
  const PersistArgs& A = *c.A;
  Misc* ms = c.ms;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (lane == 0) ms->wbest[wid] = best;
  consumer_sync();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < NCW; ++w) b = umax64(b, ms->wbest[w]);
    A.am_part[blockIdx.x] = b;
    __threadfence();
    ms->last = (atomicAdd(A.head_cnt, 1) == (int)gridDim.x - 1);
  }
  consumer_sync();
  if (ms->last) {
    __threadfence();
    unsigned long long b = 0ull;
    for (int q = threadIdx.x; q < (int)gridDim.x; q += PT) b = umax64(b, __ldcg(A.am_part + q));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) b = umax64(b, __shfl_xor_sync(0xffffffffu, b, o));
    if (lane == 0) ms->wbest[wid] = b;
    consumer_sync();
    if (threadIdx.x == 0) {
      for (int w = 0; w < NCW; ++w) b = umax64(b, ms->wbest[w]);
      if constexpr (TP) b = tp_argmax(c, b);
      const int step = ms->step;
      if (step < A.max_steps) A.ids[step] = am_index(b);
      else atomicCAS(A.err, 0, ERR_CTX);
      *A.head_cnt = 0;
      A.io[0] = step + 1;
      A.dyn->pos = ms->pos + 1;
      A.dyn->T = ms->T + 1;
      A.dyn->conv_base = ms->conv_base + 1;
      A.dyn->seq = ms->seq + 1;
    }
  }
}

// ---------------------------------------------------------------- tensor-core head
//
// The tied head (248320 x HID) runs on tcgen05.mma kind::i8.  A CTA's head
// tiles (128 embedding rows x HID) stream through the ring as 16 KB K-slabs.
// Roles:
//   warp NCW-1 lane 0  issues, per slab, four K = 32 MMAs (M = 128 rows of A =
//                      the slab, N = 16 rows of B = the x digit planes) into
//                      a double-buffered TMEM accumulator (columns 16 (T & 1)
//                      .. +15, T = the CTA's running tile count);
//   warp NCW-2 lane 0  refills each slab's slot once its MMAs have completed;
//   warps 0-3          epilogue: thread = TMEM lane = tile row, the three exact
//                      digit sums recombined and scaled exactly as the CUDA-core
//                      GEMVs do (finish_f32), logits stored, argmax kept.


// Refiller (one thread) over the phase's slabs [i0, i1): wait for the MMAs of
// slab q (per-slot commit parity in *mpar), release its slot on the empty
// barrier and issue chunk q + NSLOT into it.  1 = ok.
__device__ int tile_refill(PCtx& c, int i0, int i1, unsigned& mpar) {
  for (int q = i0; q < i1; ++q) {
    const int s = q % NSLOT;
    if (!wait_bar1(c, mma_bar(c, s), (mpar >> s) & 1u, 15, q)) return 0;
    mpar ^= 1u << s;
    const int nx = q + NSLOT;
    if (nx < c.nch) {
      // (the head is the last phase: no chunk after it waits on the slot's
      // empty barrier, so the refill goes out as soon as the MMAs are done)
      issue_chunk(c, nx);
      c.ms->slot_last[s] = nx;
    }
  }
  return 1;
}

// MMA issuer (one thread) over the phase's slabs [i0, i1); T0 = tiles this CTA
// issued earlier in the step.  A tile's buffer is reused once the epilogue
// released the tile two before it.  1 = ok.
__device__ int tile_mma(PCtx& c, int i0, int i1, unsigned tmem, int T0) {
  constexpr unsigned IDESC = umma_idesc_i8(HEAD_TM, 16);
  constexpr unsigned SBO_A = (HEAD_KS / 16) * 128;
  const unsigned bt = smem_u32(c.sm + OFF_BT);
  const unsigned s_lo = smem_u32(c.sm), s_hi = s_lo + SMEM_BYTES;
  // the accumulators: lane 0, two 16-column buffers inside the 512 columns
  if ((tmem >> 16) != 0u || (tmem & 0xffffu) > 512u - 32u) { check_fail(c, 2, (int)tmem); return 0; }
  if (bt < s_lo || bt + 2u * BT_SBO > s_hi) { check_fail(c, 4, (int)bt); return 0; }
  if (i1 > i0) c.ms->mma_any = 1;
  // descriptors: slot 0 / B tile at slab 0; a K = 32 step adds 256 B to both
  const unsigned long long da0 = umma_desc(smem_u32(c.sm + OFF_RING), 128u, SBO_A);
  const unsigned long long db0 = umma_desc(bt, 128u, (unsigned)BT_SBO);
  for (int i = i0; i < i1; ++i) {
    const int li = i - i0, t = T0 + li / HEAD_NSLAB, j = li % HEAD_NSLAB, b = t & 1;
    if (j == 0 && t >= 2) {
      if (!wait_bar1(c, acce_bar(c, b), (unsigned)(((t - 2) >> 1) & 1), 13, t)) return 0;
      tc_fence_after();
    }
    if (!wait_bar1(c, full_bar(c, i % NSLOT), (unsigned)((i / NSLOT) & 1), 14, i)) return 0;
    const unsigned a = smem_u32(c.sm + OFF_RING + (i % NSLOT) * SLOT);
    if (a < s_lo || a + (unsigned)SLOTW > s_hi || (a & 127u)) { check_fail(c, 3, (int)a); return 0; }
    // start-address fields are addr >> 4 in the low 14 bits (no carry: smem < 256 KB)
    const unsigned long long da = da0 + (unsigned long long)(((i % NSLOT) * SLOT) >> 4);
    const unsigned long long db = db0 + (unsigned long long)((HEAD_KS / 16) * j * 8);
    const unsigned dt = tmem + 16u * b;
    umma_i8(dt, da, db, IDESC, (unsigned)j);
    umma_i8(dt, da + 16, db + 16, IDESC, 1u);
    umma_i8(dt, da + 32, db + 32, IDESC, 1u);
    umma_i8(dt, da + 48, db + 48, IDESC, 1u);
    umma_commit(mma_bar(c, i % NSLOT));
    if (j == HEAD_NSLAB - 1) umma_commit(accf_bar(c, b));
  }
  return 1;
}

// The tied head on the tensor cores: chunks [i0, i1) are this CTA's head tile
// slabs (possibly none: the argmax merge still needs every CTA).  Input: the
// residual stream after the last layer, final-normed, encoded once into the B
// tile.
template <bool TP>
__device__ bool phase_head(PCtx& c, int p, int i0, int i1) {
  const PersistArgs& A = *c.A;
  Misc* ms = c.ms;
  float* hs = (float*)(c.sm + OFF_HS);
  const float2 g2 = __ldg(reinterpret_cast<const float2*>(A.final_norm) + threadIdx.x);
  if (!wait_tagged(c, A.tv_h, HID, tag_of(c, p - 1), hs)) return false;
  trace_mark(c, p, 1);
  float inv, sx;
  cta_encode_1024(c, hs, g2, false, inv, sx, true);
  const float xsf = (float)ms->scale;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int ntiles = (i1 - i0) / HEAD_NSLAB;
  const int T0 = ms->ntile;
  const unsigned tmem = ms->tmem;
  const bool want = ms->want_logits != 0;
  unsigned long long best = 0ull;
  int good = 1;
  if ((i1 - i0) % HEAD_NSLAB != 0 || (ntiles > 0 && !(c.ch[i0].seg & CHUNK_MMA))) {
    if (threadIdx.x == 0) check_fail(c, 1, i1 - i0);
    good = 0;
  }
  if (!good || ntiles == 0) {
  } else if (wid == NCW - 1) {
    if (lane == 0) good = tile_mma(c, i0, i1, tmem, T0);
    __syncwarp();
  } else if (wid == NCW - 2) {
    if (lane == 0) {
      unsigned mpar = ms->mpar;
      good = tile_refill(c, i0, i1, mpar);
      ms->mpar = mpar;
    }
    __syncwarp();
  } else if (wid < 4) {
    for (int tl = 0; tl < ntiles; ++tl) {
      const int T = T0 + tl, b = T & 1;
      const int o = (int)c.ch[i0 + tl * HEAD_NSLAB].row0 * HEAD_TM + 32 * wid + lane;   // TMEM lane = tile row
      if (__any_sync(0xffffffffu, o >= VOCAB)) {
        if (lane == 0) check_fail(c, 6, o);
        good = 0;
        break;
      }
      const float sw = __ldg(A.emb_s + o);
      if (!wait_bar_warp(c, accf_bar(c, b), (unsigned)((T >> 1) & 1), 17, T)) { good = 0; break; }
      if (tl == 0) trace_mark(c, p, 2);
      tc_fence_after();
      // this warp's 32 TMEM lanes (rows), columns 0-2 (the digit sums)
      const unsigned ta = tmem + ((unsigned)(32 * wid) << 16) + 16u * b;
      unsigned r0, r1, r2;
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];"
                   : "=r"(r0), "=r"(r1) : "r"(ta) : "memory");
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r2) : "r"(ta + 2u) : "memory");
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(c, b));
      const float y = finish_f32((int)r0, (int)r1, (int)r2, 3, xsf * sw);
      if (want) A.logits[o] = y;
      best = umax64(best, am_pack(y, o));
    }
  }
  if (!consumer_and(good)) return false;
  if (threadIdx.x == 0) { ms->ntile = T0 + ntiles; ms->hs_tag = 0; }
  head_finish<TP>(c, best);
  return true;
}

// ---------------------------------------------------------------- panel GEMVs
//
// The layer projections run on the warp-level tensor-core MMA, mma.sync
// m16n8k32 s8 x s8 -> s32 (exact): A = 16 panel rows x 32 K (one ldmatrix.x4;
// the panel layout makes a K-step 512 contiguous bytes), B = the x digits
// (column d = digit d, the other columns zero) from the fragment-ordered digit
// image.  A chunk splits into tasks of 4 KB of weights -- 8 K-steps of a plain
// chunk, or 4 gate + 4 up K-steps of a pair chunk; an fp32 chunk splits into
// one task per row.  Task t of a phase runs on warp t % NCW and adds its digit
// sums into the panel's accumulators in shared memory (int32 adds: exact, so
// their order does not matter).

__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned (&a)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ void mma_s8(int (&d)[4], const unsigned (&a)[4], uint2 b) {
  asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}
__device__ __forceinline__ void red_add_s32(unsigned addr, int v) {
  asm volatile("red.shared.add.s32 [%0], %1;" :: "r"(addr), "r"(v) : "memory");
}

// Digit sums of the 16 rows of a panel over ns K-steps (a multiple of 4): A at
// shared address a (K-step s at a + 512 s), B from the digit image fr at
// K-step s0, nd digits (B columns nd.. read as zero); two accumulator chains
// (even / odd steps).  The m16n8 accumulator fragment has rows g, g + 8 of
// columns 2u, 2u + 1 in lane (g, u) = (lane / 4, lane % 4); it comes back
// rearranged: lane u = 0 holds digits 0-2 of row g, lane u = 1 those of row
// g + 8, lanes u = 2, 3 nothing.  One body for every GEMV phase and digit
// count, so the phases share its instructions.
__device__ __forceinline__ void panel_mma(unsigned a, const unsigned char* fr, int s0, int ns, int nd,
                                          int (&d3)[3]) {
  const int lane = threadIdx.x & 31;
  int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
  a += 16u * lane;
  const unsigned char* fb = fr + 96 * s0 + 8 * lane;
  const bool bl = lane < 4 * nd;
#pragma unroll 1
  for (int s = 0; s < ns; s += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      unsigned w[4];
      ldsm_x4(a + 512u * (s + u), w);
      const uint2 b = bl ? *reinterpret_cast<const uint2*>(fb + 96 * (s + u)) : make_uint2(0u, 0u);
      if (u & 1) mma_s8(c1, w, b);
      else mma_s8(c0, w, b);
    }
  }
  int c[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) c[e] = c0[e] + c1[e];
  const int u = lane & 3;
  const int x = __shfl_xor_sync(0xffffffffu, u == 0 ? c[2] : c[0], 1);
  const int y = __shfl_xor_sync(0xffffffffu, c[3], 1);
  d3[0] = u == 0 ? c[0] : x;
  d3[1] = u == 0 ? c[1] : y;
  d3[2] = u == 0 ? x : c[2];
}

// Tasks of chunk k of a GEMV phase with K window kw (kwin_of): a panel
// slice's K in pieces of at most TASK_KB (multiples of 128).
__host__ __device__ __forceinline__ int chunk_tasks(const Chunk& k, unsigned kw) {
  if (!(k.seg & CHUNK_PANEL)) return k.nrows;
  const int rem = (int)(kw >> 16) - (int)(kw & 0xffffu) - (int)k.nrows * PANEL_KB;
  return ((rem < PANEL_KB ? rem : PANEL_KB) + TASK_KB - 1) / TASK_KB;
}

// Task map of a GEMV phase over chunks [i0, i0 + nj), nj <= NSLOT, held in
// registers by every warp (lane = chunk): nq = the chunk's tasks, tb / pv =
// inclusive prefix sums of tasks / panel starts over the chunks.  Task t lies
// in the first chunk whose tb exceeds t; panel v starts at the chunk whose pv
// is v + 1.  Every warp runs exactly its own tasks (t = wid, wid + NCW, ...).
struct TaskMap {
  int nq, tb, pv, start, pan, ntask, npan;
};
__device__ __forceinline__ TaskMap task_map(const PCtx& c, unsigned kw, int i0, int nj) {
  const int lane = threadIdx.x & 31;
  TaskMap m;
  m.nq = 0;
  m.start = 0;
  m.pan = 0;
  if (lane < nj) {
    const Chunk k = c.ch[i0 + lane];
    m.nq = chunk_tasks(k, kw);
    if (k.seg & CHUNK_PANEL) {
      m.pan = 1;
      m.start = 1;
      if (lane > 0) {
        const Chunk kp = c.ch[i0 + lane - 1];
        if ((kp.seg & CHUNK_PANEL) && kp.row0 == k.row0) m.start = 0;
      }
    }
  }
  m.tb = m.nq;
  m.pv = m.start;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, m.tb, o), b = __shfl_up_sync(0xffffffffu, m.pv, o);
    if (lane >= o) { m.tb += a; m.pv += b; }
  }
  m.ntask = __shfl_sync(0xffffffffu, m.tb, 31);
  m.npan = __shfl_sync(0xffffffffu, m.pv, 31);
  return m;
}
// chunk (of the phase) holding task t < ntask, and t's K-part within it
__device__ __forceinline__ int task_chunk(const TaskMap& m, int t, int& q) {
  const int j = __ffs(__ballot_sync(0xffffffffu, m.tb > t)) - 1;
  q = t - __shfl_sync(0xffffffffu, m.tb - m.nq, j);
  return j;
}
// panel (of the phase) of chunk j
__device__ __forceinline__ int chunk_panel(const TaskMap& m, int j) {
  return __shfl_sync(0xffffffffu, m.pv, j) - 1;
}
// first chunk of panel v < npan
__device__ __forceinline__ int panel_chunk(const TaskMap& m, int v) {
  return __ffs(__ballot_sync(0xffffffffu, m.start && m.pv == v + 1)) - 1;
}
// Row scale of row pr of panel q of GEMV phase `sub` (a pair panel: rows 0-7
// gate rows 8q.., rows 8-15 the same up rows).
__device__ __forceinline__ const float* row_scale(const LayerW& L, int sub, int q, int pr) {
  if (sub == 3) return (pr < PAIR_ROWS ? L.gate_s : L.up_s) + q * PAIR_ROWS + pr % PAIR_ROWS;
  const int r = q * PANEL + pr;
  if (sub == 0) {
    if (L.linear) return r < CONVD ? L.qkv_s + r : L.z_s + (r - CONVD);
    return r < QPROJ ? L.q_s + r : (r < QPROJ + KVPROJ ? L.k_s + (r - QPROJ) : L.v_s + (r - QPROJ - KVPROJ));
  }
  return (sub == 2 ? (L.linear ? L.out_s : L.o_s) : L.down_s) + r;
}

// Row-parallel OUT / DOWN under tensor parallelism: the 16 residual rows of
// panel q (lane = row pr, own lanes; hres = the lane's residual value) once
// every rank's partial of them is in this rank's exchange buffer xb
// ([TP_MAX][HID] of the phase kind), h = r + ((y_0 + y_1) + ...) in rank
// order (bit-identical on every rank),
// written as tagged words to tv_h.  One warp.  Bounded wait; false on abort.
// Not inlined, plain arguments: only tensor-parallel runs execute it.
__device__ __noinline__ bool tp_reduce_panel(const unsigned long long* xb, unsigned long long* tv_h, float hres,
                                             int q, int P, bool own, int pr, unsigned tag, Misc* ms, int* err,
                                             int* abort_flag, int sub) {
  const int lane = threadIdx.x & 31;
  const int r = q * PANEL + pr;
  const unsigned long long t0 = gtime();
  int it = 0;
  float sum = 0.0f;
  bool done = !own;
  for (;;) {
    if (!done) {
      bool all = true;
      for (int rr = 0; rr < P && all; ++rr) all = tag_ok(ld_tv_sys(xb + (size_t)rr * HID + r), tag);
      if (all) {
        sum = tv_val(ld_tv_sys(xb + r));
        for (int rr = 1; rr < P; ++rr) sum = __fadd_rn(sum, tv_val(ld_tv_sys(xb + (size_t)rr * HID + r)));
        done = true;
      }
    }
    if (__all_sync(0xffffffffu, done)) break;
    if (((++it) & 63) == 0) {
      int bad = 0;
      if (lane == 0) {
        if (*(volatile int*)&ms->abort || ld_flag(abort_flag)) {
          bad = 1;
        } else if (gtime() - t0 > WAIT_NS) {
          record_error(err, abort_flag, ms, ERR_WAIT, 23, sub);
          bad = 1;
        }
      }
      if (__shfl_sync(0xffffffffu, bad, 0)) return false;
    }
  }
  if (own) st_tv(tv_h + r, __fadd_rn(hres, sum), tag);
  return true;
}

// mma.m16n8k32 with signed int8 A (weights) and unsigned int8 B (digits).
__device__ __forceinline__ void mma_s8u8(int (&d)[4], const unsigned (&a)[4], uint2 b) {
  asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}
// Sums of the 16 rows of a panel over ns K-steps (a multiple of 4) of a
// slice: A at shared address a (K-step s at a + 512 s), B = the slice's three
// unsigned digit planes (columns 0-2, from the image fr in the B-fragment
// order of dig_off) and a column of ones (column 3: the rows' weight sums);
// four independent accumulator chains.  Lane u = 0 returns row g's S0, S1,
// S2, Sw (g = lane / 4), lane u = 1 row g + 8's; lanes u = 2, 3 nothing.
__device__ __forceinline__ void slice_mma(unsigned a, const unsigned char* fr, int ns, int (&d4)[4]) {
  const int lane = threadIdx.x & 31;
  int c[4][4];
#pragma unroll
  for (int u = 0; u < 4; ++u) c[u][0] = c[u][1] = c[u][2] = c[u][3] = 0;
  a += 16u * lane;
  const unsigned char* fb = fr + 8 * lane;
  const bool dig = lane < 12;
  const uint2 ones = lane < 16 ? make_uint2(0x01010101u, 0x01010101u) : make_uint2(0u, 0u);
#pragma unroll 1
  for (int s = 0; s < ns; s += 4) {
    unsigned w[4][4];
    uint2 b[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      ldsm_x4(a + 512u * (s + u), w[u]);
      b[u] = dig ? *reinterpret_cast<const uint2*>(fb + 96 * (s + u)) : ones;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) mma_s8u8(c[u], w[u], b[u]);
  }
  int r[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) r[e] = (c[0][e] + c[1][e]) + (c[2][e] + c[3][e]);
  const int u = lane & 3;
  const int x = __shfl_xor_sync(0xffffffffu, u == 0 ? r[2] : r[0], 1);
  const int y = __shfl_xor_sync(0xffffffffu, u == 0 ? r[3] : r[1], 1);
  d4[0] = u == 0 ? r[0] : x;
  d4[1] = u == 0 ? r[1] : y;
  d4[2] = u == 0 ? x : r[2];
  d4[3] = u == 0 ? y : r[3];
}

// Ring slots a warp refills at the top of the next phase: up to two runs of
// chunks were fully read (Misc::rfq[warp]: first | count << 16); chunk + NSLOT
// goes into each one's slot.
__device__ __forceinline__ void note_refill(Misc* ms, int a, int n) {
  int* q = ms->rfq[threadIdx.x >> 5];
  if ((threadIdx.x & 31) == 0) q[q[0] != 0] = a | n << 16;
  __syncwarp();
}
__device__ __forceinline__ void do_refills(PCtx& c) {
  const int lane = threadIdx.x & 31;
  int* q = c.ms->rfq[threadIdx.x >> 5];
  for (int r = 0; r < 2; ++r) {
    const int a = q[r] & 0xffff, n = q[r] >> 16;
    if (lane < n) {
      const int ii = a + lane, nx = ii + NSLOT;
      if (nx < c.nch && !*(volatile int*)&c.ms->abort) {
        issue_chunk(c, nx);
        c.ms->slot_last[ii % NSLOT] = nx;
      }
    }
  }
  __syncwarp();
  if (lane == 0) q[0] = q[1] = 0;
  __syncwarp();
}

// A GEMV phase over panels (IN, OUT, GATEUP, DOWN).
//   Before the input arrives, warp v < npan stages panel v's row scales in
//   shared memory and every warp waits for its first task's chunk.
//   The input vector is then encoded once into the CTA's digit image:
//     W8A32 (default): the input wait folds max|v| of the values as they
//     arrive (v = z = h * (1 + w) for the normed input of IN / GATEUP, else x)
//     and, for a normed input, each warp's sum of h^2; one barrier after the
//     wait (encode_fixed) completes the image.  The 1/rms
//     (golden/model.py:63-75) is applied with 2^-shift when a panel finishes.
//     ACT_INT8: the golden per-vector quantiser of x itself (cta_encode_1024,
//     encode_lin).
//   Task t runs on warp t % NCW and adds exact int32 digit sums into its
//   panel's accumulators.  The warp that completes a panel's last task
//   finishes the panel -- the projection rows (IN), silu(gate) * up (GATEUP,
//   golden/model.py:236), or h + y (OUT, DOWN; under TP the partial rows are
//   exchanged first) -- and refills the panel's ring slots.  No CTA barrier
//   between tasks and outputs.
// Every piece of the phase's code appears once (one wait, one encode), so a
// GEMV CTA's instruction working set stays small.  (The fp32 in_proj_b /
// in_proj_a rows of a DeltaNet IN are dotted by the heads' own CTAs,
// gate_inputs.)
template <bool TP, bool I8, bool NORMED>
__device__ bool phase_panels(PCtx& c, int p, int i0, int i1) {
  const PersistArgs& A = *c.A;
  Misc* ms = c.ms;
  float* hs = (float*)(c.sm + OFF_HS);
  float* xf = (float*)(c.sm + OFF_XF);
  float* zb = (float*)(c.sm + OFF_DIG);   // silu(z) of the gated norm, parked in the digit region
  const int l = p / 5, sub = p % 5;
  const LayerW& L = c.lay[l];
  constexpr bool normed = NORMED;   // IN, GATEUP (else OUT, DOWN)
  const bool gated = sub == 2 && L.linear;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nj = i1 - i0;
  trace_warp(c, p, 0);
  int good = 1;
  if (nj > NSLOT) {   // the schedule keeps a phase within the ring (MAXPAN panels)
    if (threadIdx.x == 0) check_fail(c, 8, nj);
    good = 0;
  }
  const unsigned kw = kwin_t<TP>(A, sub);
  const TaskMap m = task_map(c, kw, i0, good ? nj : 0);
  const int tpp = m.npan > 0 ? m.ntask / m.npan : 1;      // tasks per panel (same window for all)
  const int cpp = m.npan > 0 ? nj / m.npan : 1;           // chunks per panel
  // panel row of this lane in the finishing step (lanes with lane & 2 hold none)
  const bool own = (lane & 2) == 0;
  const int pr = (lane >> 2) + 8 * (lane & 1);
  float* psc = (float*)(c.sm + OFF_PSC);
  if (wid < m.npan) {
    const int fc = panel_chunk(m, wid);   // (a warp collective: every lane)
    if (lane < PANEL) psc[wid * PANEL + lane] = __ldg(row_scale(L, sub, (int)c.ch[i0 + fc].row0, lane));
  }
  const float2 g2 = normed ? __ldg(reinterpret_cast<const float2*>(sub == 0 ? L.in_norm : L.post_norm) + threadIdx.x)
                           : make_float2(0.f, 0.f);
  const float gwn = gated ? __ldg(L.gnorm_w + (threadIdx.x % LV)) : 0.0f;
  // the first task's chunk (requested in an earlier phase, so waiting for it
  // here cannot hold anything up)
  bool first_in = false;
  if (good && wid < m.ntask) {
    int q;
    first_in = wait_full(c, i0 + task_chunk(m, wid, q));
    if (!first_in) good = 0;
    trace_warp(c, p, 3);
  }
  // The inputs, polled together.  Normed (IN, GATEUP): the residual stream h
  // (golden/model.py:142,262) into hs.  OUT (sub 2) and DOWN (sub 4): the
  // projection's input -- the delta-rule output o (DeltaNet OUT, gated
  // below), the gated attention output o * sigmoid(gate) written by the merge
  // (attention OUT), or silu(gate) * up (DOWN) -- over the phase's K window
  // [k0, k1) (kwin: all of it, or the rank's columns under tensor
  // parallelism) into xf at its positions; for the gated norm silu(z) of the
  // window (IN(l) wrote it); and the residual stream the projection is added
  // to (golden/model.py:259,263), unless hs holds it already.  Layer 0 starts
  // from the dequantised embedding row (golden/model.py:246).
  unsigned* amax = I8 ? nullptr : &ms->amax[p & 1];
  const int k0 = normed ? 0 : (int)(kw & 0xffffu), k1 = normed ? HID : (int)(kw >> 16);
  const unsigned need = tag_of(c, normed ? p - 1 : (p == 2 ? -1 : (sub == 4 ? p - 2 : p - 3)));
  const bool embed = need == tag_of(c, -1) && ms->hs_tag != need;   // layer 0: the embedding row into hs
  if (embed) {
    const int tok = ms->tok;
    const float sc = __ldg(A.emb_s + tok);
    const int8_t* row = A.emb_q + (size_t)tok * HID;
    for (int i = threadIdx.x; i < HID; i += PT) hs[i] = __fmul_rn((float)row[i], sc);
  }
  const bool need_h = !embed && ms->hs_tag != need;
  if constexpr (NORMED) {
    const WSeg sh{A.tv_h, hs, need_h ? HID / 2 : 0, need}, none{A.tv_h, hs, 0, 0u};
    if (!wait_inputs(ms, A.err, A.abort_flag, sh, none, none, amax, true, g2, I8 ? nullptr : ms->ssw))
      return false;
  } else {
    const unsigned long long* src = sub == 4 ? A.tv_act : (L.linear ? A.tv_o : A.tv_attn);
    const WSeg sx_{src + k0, xf + k0, (k1 - k0) / 2, tag_of(c, p - 1)};
    const WSeg sz{A.tv_z + k0, zb + k0, gated ? (k1 - k0) / 2 : 0, tag_of(c, p - 2)};
    const WSeg sr{A.tv_h, hs, need_h ? HID / 2 : 0, need};
    if (!wait_inputs(ms, A.err, A.abort_flag, sx_, sz, sr, gated ? nullptr : amax, false, make_float2(0.f, 0.f),
                     nullptr))
      return false;
  }
  if (embed && normed && amax) {
    // (the embedding row did not pass through the wait: fold it here)
    const float h0 = hs[2 * threadIdx.x], h1 = hs[2 * threadIdx.x + 1];
    const float vm = fmaxf(fabsf(__fmul_rn(h0, __fadd_rn(1.0f, g2.x))), fabsf(__fmul_rn(h1, __fadd_rn(1.0f, g2.y))));
    const unsigned wm = __reduce_max_sync(0xffffffffu, __float_as_uint(vm));
    if (lane == 0 && wm) asm volatile("red.shared.max.u32 [%0], %1;" :: "r"(smem_u32(amax)), "r"(wm) : "memory");
    const float ss = warp_sum(fmaf(h1, h1, __fmul_rn(h0, h0)));
    if (lane == 0) ms->ssw[wid] = ss;
    consumer_sync();
  }
  if (threadIdx.x == 0) ms->hs_tag = need;
  trace_warp(c, p, 1);
  if (gated) {
    // gated RMSNorm of the delta-rule output (golden/model.py:183-189) over the
    // window's heads
    for (int h = k0 / LV + wid; h < k1 / LV; h += NCW) {
      float ss = 0.0f;
      for (int i = lane; i < LV; i += 32) ss = fmaf(xf[h * LV + i], xf[h * LV + i], ss);
      ss = warp_sum(ss);
      // (ss / LV: LV is a power of two, so the product by 1/LV is the same number)
      if (lane == 0) ms->inv_h[h] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / LV), EPS)));
    }
    consumer_sync();
    float vmax = 0.0f;
    for (int i = k0 + threadIdx.x; i < k1; i += PT) {
      const float v = __fmul_rn(__fmul_rn(xf[i], ms->inv_h[i / LV]), gwn);
      xf[i] = __fmul_rn(v, zb[i]);
      vmax = fmaxf(vmax, fabsf(xf[i]));
    }
    if (amax) {
      const unsigned wm = __reduce_max_sync(0xffffffffu, __float_as_uint(vmax));
      if (lane == 0 && wm) asm volatile("red.shared.max.u32 [%0], %1;" :: "r"(smem_u32(amax)), "r"(wm) : "memory");
    }
    consumer_sync();
  }
  trace_mark(c, p, 1);
  // W8A8 capture: the first CTA to reach the phase records its input
  bool dbg_cta = false;
  if constexpr (I8 && !TP) {
    if (p == A.dbg_phase) {
      if (threadIdx.x == 0) ms->last = atomicCAS((int*)(A.dbg + DBG_FLAG), 0, 1) == 0;
      consumer_sync();
      dbg_cta = ms->last != 0;
      if (dbg_cta)
        for (int e = threadIdx.x; e < k1; e += PT) A.dbg[DBG_X + e] = normed ? hs[e] : xf[e];
    }
  }
  // the digit image
  float sx = 0.0f, xs = 0.0f;
  if constexpr (I8) {
    if (normed) {
      float inv;
      cta_encode_1024(c, hs, g2, true, inv, sx, false, p);
    } else if constexpr (TP) {
      if (!tp_encode_i8(c, p, k0, k1)) return false;
    } else {
      encode_lin(c, k1, true);
    }
  } else {
    if constexpr (NORMED) xs = encode_u8(c.sm, hs, 0, HID, *amax, sub == 0 ? L.in_norm : L.post_norm);
    else xs = encode_u8(c.sm, xf, k0, k1, *amax, nullptr);
    // every thread has read amax: re-arm it for phase p + 2
    if (threadIdx.x == 0) *amax = 0u;
  }
  trace_warp(c, p, 2);
  if (dbg_cta) {
    const int8_t* dg = (const int8_t*)(c.sm + OFF_DIG);
    for (int e = threadIdx.x; e < k1; e += PT) A.dbg[DBG_XQ + e] = (float)dg[dig_off(0, e & ~3) + (e & 3)];
    if (threadIdx.x == 0) { A.dbg[DBG_SX] = (float)ms->scale; A.dbg[DBG_K] = (float)k1; }
  }
  // x scale of the digit sums: ACT_INT8 the quantiser's s_x; W8A32 2^-shift,
  // times 1/rms for a normed input (exact: a power of two times a float), the
  // rms from the warps' sums of h^2 (golden/model.py:74: mean over HID)
  float xsc = xs;
  if constexpr (I8) {
    xsc = (float)ms->scale;
  } else if (normed) {
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) tot = __fadd_rn(tot, ms->ssw[w]);
    // tot / HID as the product by 1/HID (HID a power of two: the same number);
    // 1/sqrt through the correctly rounded reciprocal
    xsc = __fmul_rn(xs, __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(tot, 1.0f / HID), EPS))));
  }
  const unsigned char* fr = c.sm + OFF_DIG;                   // the CTA's digit image
  const unsigned part = smem_u32(c.sm + OFF_PART);
  const int nd = I8 ? ms->ndig : 3;   // (W8A32: three unsigned digits and the weight sums)
  const unsigned tag = tag_of(c, p);
  for (int t = wid; good && t < m.ntask; t += NCW) {
    int q;
    const int j = task_chunk(m, t, q);
    const int i = i0 + j;
    const Chunk k = c.ch[i];
    if (!(k.seg & CHUNK_PANEL)) {
      if (lane == 0) check_fail(c, 9, i);
      good = 0;
      break;
    }
    if (!(t == wid && first_in) && !wait_full(c, i)) { good = 0; break; }
    const int kb = k0 + (int)k.nrows * PANEL_KB + TASK_KB * q;   // the task's first K position
    const unsigned sa = smem_u32(c.sm + OFF_RING + (i % NSLOT) * SLOT) + 512u * (TASK_KB / 32) * q;
    // task length: a multiple of 128; whole inputs (every K a multiple of TASK_KB) always TASK_KB
    const int kl = !TP ? TASK_KB : (k1 - kb < TASK_KB ? k1 - kb : TASK_KB);
    int d4[4];
    if constexpr (I8) {
      int d3[3];
      panel_mma(sa, fr, kb >> 5, kl >> 5, nd, d3);
      d4[0] = d3[0];
    } else {
      slice_mma(sa, fr + 96 * (kb >> 5), kl >> 5, d4);
    }
    trace_warp(c, p, 5);
    const int vp = chunk_panel(m, j);
    if (own) {
      const unsigned pv = part + 4u * (unsigned)(vp * 4 * PANEL + pr);
      red_add_s32(pv, d4[0]);
      if constexpr (!I8) {
        red_add_s32(pv + 4u * PANEL, d4[1]);
        red_add_s32(pv + 8u * PANEL, d4[2]);
        red_add_s32(pv + 12u * PANEL, d4[3]);
      }
    }
    // the last of the panel's tasks finishes it
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atom_add_acq_rel_cta(&ms->pcnt[vp], 1) == tpp - 1;
    if (!__shfl_sync(0xffffffffu, last, 0)) continue;
    const int fc = panel_chunk(m, vp);    // the panel's first chunk (a warp collective)
    const int pq = (int)c.ch[i0 + fc].row0;
    float y = 0.0f;
    if (own) {
      // the panel's exact sums, and the accumulators zeroed for the next phase
      int* pvp = (int*)(c.sm + OFF_PART) + vp * 4 * PANEL + pr;
      if constexpr (I8) {
        y = finish_f32(pvp[0], 0, 0, 1, xsc * psc[vp * PANEL + pr]);
        if constexpr (!TP) {
          if (p == A.dbg_phase) {   // the row's accumulator (GATEUP: gate rows, then up rows)
            const int rr = sub == 3 ? (pr < PAIR_ROWS ? pq * PAIR_ROWS + pr : FFN + pq * PAIR_ROWS + pr - PAIR_ROWS)
                                    : pq * PANEL + pr;
            reinterpret_cast<int*>(A.dbg)[DBG_ACC + rr] = pvp[0];
          }
        }
        pvp[0] = 0;
      } else {
        // the row's exact sum of w * X: sum of w * U minus 2^22 times the weight sum
        const double xsum = fma((double)pvp[2 * PANEL], 65536.0, fma((double)pvp[PANEL], 256.0, (double)pvp[0])) -
                            4194304.0 * (double)pvp[3 * PANEL];
        y = (float)(xsum * (double)(xsc * psc[vp * PANEL + pr]));
        pvp[0] = 0;
        pvp[PANEL] = 0;
        pvp[2 * PANEL] = 0;
        pvp[3 * PANEL] = 0;
      }
    }
    if (lane == 0) ms->pcnt[vp] = 0;
    if (sub == 3) {
      // pair panel: lane pr = g holds gate row 8q + g, its neighbour the up row
      const float up = __shfl_xor_sync(0xffffffffu, y, 1);
      if (own && (lane & 1) == 0) st_tv(A.tv_act + pq * PAIR_ROWS + pr, __fmul_rn(silu_f(y), up), tag);
    } else if (own) {
      const int r = pq * PANEL + pr;
      if (sub == 0) {
        unsigned long long* out;
        int o;
        if (L.linear) {
          if (r < CONVD) { out = A.tv_qkv; o = r; }
          else { out = A.tv_z; o = r - CONVD; y = silu_f(y); }   // the gated norm of OUT takes silu(z)
        } else {
          if (r < QPROJ) { out = A.tv_qg; o = r; }
          else if (r < QPROJ + KVPROJ) { out = A.tv_kvn; o = r - QPROJ; }
          else { out = A.tv_kvn + KVPROJ; o = r - QPROJ - KVPROJ; }
        }
        st_tv(out + o, y, tag);
      } else if constexpr (!TP) {
        st_tv(A.tv_h + r, __fadd_rn(hs[r], y), tag);
      } else {
        // row-parallel: this rank's partial row into every rank's exchange buffer
        const size_t off = XB_PART + ((size_t)(sub == 4) * TP_MAX + A.tp_rank) * HID + r;
        for (int rr = 0; rr < A.tp_world; ++rr) st_tv_sys(A.xbuf[rr] + off, y, tag);
      }
    }
    if constexpr (TP) {
      if (sub == 2 || sub == 4) {
        if (!tp_reduce_panel(A.xbuf[A.tp_rank] + XB_PART + (size_t)(sub == 4) * TP_MAX * HID, A.tv_h, hs[pq * PANEL + pr], pq,
                             A.tp_world, own, pr, tag, ms, A.err, A.abort_flag, sub)) {
          good = 0;
          break;
        }
      }
    }
    // the panel's outputs are out: its slots can be refilled (every task that
    // read them has finished).  The refill is left to the top of the next
    // phase (the bulk-copy issue can wait for the copy engine), so that this
    // warp reaches the phase's end at once.
    trace_warp(c, p, 6);
    if (lane == 0) trace_latest(c, p, 2);
    note_refill(ms, i0 + fc, cpp);
  }
  trace_warp(c, p, 4);
  return good != 0;
}

// ---------------------------------------------------------------- DeltaNet heads
//
// Every DeltaNet head has its own CTA (CTA h - h0 for the rank's heads
// [h0, h1)), which runs no GEMV panel: during IN it computes the head's gate
// inputs, during MIX the head's conv, gates, l2norm and delta rule.

// IN phase of linear layer l on head h's CTA: b = in_proj_b[h] . x and
// a = in_proj_a[h] . x (fp32 rows, golden/model.py:146-147) with x the normed
// layer input (golden/model.py:142; under ACT_INT8 its golden fake-quant,
// golden/model.py:37-45, 143), kept in shared memory for the head's delta
// rule in the MIX phase.  The rows are read before the input wait.
__device__ bool gate_inputs(PCtx& c, int p, int h) {
  const PersistArgs& A = *c.A;
  Misc* ms = c.ms;
  const LayerW& L = c.lay[p / 5];
  float* hs = (float*)(c.sm + OFF_HS);
  const int t = threadIdx.x;
  const bool i8 = ms->act_int8 != 0;
  const float2 g2 = __ldg(reinterpret_cast<const float2*>(L.in_norm) + t);
  const float2 wb = __ldg(reinterpret_cast<const float2*>(L.b_w + (size_t)h * HID) + t);
  const float2 wa = __ldg(reinterpret_cast<const float2*>(L.a_w + (size_t)h * HID) + t);
  if (p == 0) {
    // the residual stream starts at the dequantised embedding row (golden/model.py:246)
    const int tok = ms->tok;
    const float sc = __ldg(A.emb_s + tok);
    const int8_t* row = A.emb_q + (size_t)tok * HID;
    hs[2 * t] = __fmul_rn((float)row[2 * t], sc);
    hs[2 * t + 1] = __fmul_rn((float)row[2 * t + 1], sc);
    consumer_sync();
  } else if (!wait_tagged(c, A.tv_h, HID, tag_of(c, p - 1), hs)) {
    return false;
  }
  trace_mark(c, p, 1);
  float inv, sx;
  cta_encode_1024(c, hs, g2, i8, inv, sx);   // x (W8A8: fake-quantised) into xf[2t], xf[2t + 1]
  const float2 x = *reinterpret_cast<const float2*>(c.sm + OFF_XF + 8 * t);
  float pb = fmaf(wb.y, x.y, __fmul_rn(wb.x, x.x));
  float pa = fmaf(wa.y, x.y, __fmul_rn(wa.x, x.x));
  pb = warp_sum(pb);
  pa = warp_sum(pa);
  if ((t & 31) == 0) {
    ms->red[t >> 5] = pb;
    ms->red[NCW + (t >> 5)] = pa;
  }
  consumer_sync();
  if (t == 0) {
    float b = 0.0f, a = 0.0f;
    for (int w = 0; w < NCW; ++w) { b += ms->red[w]; a += ms->red[NCW + w]; }
    ms->abv[0] = b;
    ms->abv[1] = a;
  }
  trace_mark(c, p, 2);
  return true;
}

// MIX phase of linear layer l on head h's CTA: conv+SiLU of the head's q/k/v
// channels, gates (from gate_inputs), l2norm, the delta rule on S[h] and the
// raw o out (golden/model.py:149-178).  512 threads: 0..127 q channels,
// 128..255 k channels, 256..383 v channels, 384 the gates; the delta rule
// maps thread t to value column t % 128 and state rows 32 (t / 128) .. +31.
// Uses the digit region of smem as scratch.
__device__ bool delta_head(PCtx& c, int p, int h) {
  const PersistArgs& A = *c.A;
  Misc* ms = c.ms;
  const LayerW& L = c.lay[p / 5];
  const int t = threadIdx.x;
  const int lin = L.lin_idx;
  const int base = ms->conv_base;
  constexpr int NG = PT / LV;                                      // 4 row groups
  constexpr int KPG = LK / NG;                                     // 32 rows each
  float* qs = (float*)(c.sm + OFF_DIG);
  float* ks = qs + LK;
  float* vs = ks + LK;
  float* wsq = vs + LV;                                            // [16] per-warp sums
  float (*part)[LV] = reinterpret_cast<float (*)[LV]>(wsq + 16);  // [4][128]
  float* cs = A.conv + (size_t)lin * CONVD * CONVK;
  float* Sh = A.rec + ((size_t)lin * LH + h) * LK * LV;
  const int vi = t & (LV - 1), kg = t / LV;
  // prefetch the state, conv history and taps (previous launches wrote them)
  float sv[KPG];
#pragma unroll
  for (int kk = 0; kk < KPG; ++kk) sv[kk] = Sh[(size_t)(kg * KPG + kk) * LV + vi];
  const int role = (t < 2 * LK) ? 0 : (t < 2 * LK + LV ? 1 : (t == 2 * LK + LV ? 2 : 3));
  int ch = 0;
  if (role == 0) ch = (t < LK) ? (h * LK + t) : (KDIM + h * LK + (t - LK));
  else if (role == 1) ch = 2 * KDIM + h * LV + (t - 2 * LK);
  float s1 = 0.f, s2 = 0.f, s3 = 0.f;
  float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (role <= 1) {
    const float* st = cs + (size_t)ch * CONVK;
    s1 = st[(base + 1) & 3]; s2 = st[(base + 2) & 3]; s3 = st[(base + 3) & 3];
    w4 = *reinterpret_cast<const float4*>(L.conv_w + (size_t)ch * CONVK);
  }
  const float alog = __ldg(L.A_log + h), dtb = __ldg(L.dt_bias + h);
  // wait for this token's q/k/v projections of the head (tagged, from IN)
  const unsigned tin = tag_of(c, p - 1);
  const unsigned long long t0 = gtime();
  float nv = 0.f;
  bool have = (role >= 2);
  int it = 0;
  if (t == 0) ms->pend_min = 0x7fffffff;
  for (;;) {
    if (!have) {
      const unsigned long long w = ld_tv(A.tv_qkv + ch);
      if (tag_ok(w, tin)) { nv = tv_val(w); have = true; }
    }
    if (consumer_and(have)) break;
    if (((++it) & 15) == 0) {
      int st = 0;   // 1: aborted elsewhere, 2: this wait ran out
      if (t == 0) {
        if (aborted(c)) st = 1;
        else if (gtime() - t0 > WAIT_NS) st = 2;
      }
      if (!consumer_and(st == 0)) {
        if (!consumer_and(!(t == 0 && st == 2))) {
          // report what is missing: q/k, v, and the lowest missing channel
          if (!have) atomicMin(&ms->pend_min, ch);
          const int pq = consumer_or(!have && role == 0), pv = consumer_or(!have && role == 1);
          const int lo = (pq | pv) ? (ms->pend_min & 0x7ffff) : 0;   // a channel < CONVD
          if (t == 0) raise_abort(c, 18, p | pq << 8 | pv << 9 | lo << 12);
        }
        return false;
      }
    }
  }
  trace_mark(c, p, 1);
  float x = 0.0f;
  if (role <= 1) {
    float acc = __fmul_rn(s1, w4.x);
    acc = __fadd_rn(acc, __fmul_rn(s2, w4.y));
    acc = __fadd_rn(acc, __fmul_rn(s3, w4.z));
    acc = __fadd_rn(acc, __fmul_rn(nv, w4.w));
    x = silu_f(acc);
    cs[(size_t)ch * CONVK + (base & 3)] = nv;   // the dead oldest column takes the newest value
    if (role == 1) vs[t - 2 * LK] = x;
  } else if (role == 2) {
    ms->gate_beta = sigmoid_f(ms->abv[0]);
    ms->gate_g = __fmul_rn(-expf(alog), softplus_f(__fadd_rn(ms->abv[1], dtb)));
  }
  // l2norm of q (warps 0-3) and k (warps 4-7)
  const float ss = warp_sum(role == 0 ? x * x : 0.0f);
  if ((t & 31) == 0) wsq[t >> 5] = ss;
  consumer_sync();
  if (role == 0) {
    const int g0 = (t < LK) ? 0 : 4;
    const float tot = ((wsq[g0] + wsq[g0 + 1]) + wsq[g0 + 2]) + wsq[g0 + 3];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(tot, EPS)));
    if (t < LK) qs[t] = __fmul_rn(__fmul_rn(x, inv), 0.08838834764831845f);
    else ks[t - LK] = __fmul_rn(x, inv);
  }
  consumer_sync();
  // delta rule on the prefetched state: S *= exp(g); kv = k^T S; d = (v - kv) beta;
  // S += k (x) d; o = q^T S (after the update)
  const float gexp = expf(ms->gate_g);
  float pkv = 0.0f;
#pragma unroll
  for (int kk = 0; kk < KPG; ++kk) {
    sv[kk] = __fmul_rn(sv[kk], gexp);
    pkv = fmaf(sv[kk], ks[kg * KPG + kk], pkv);
  }
  part[kg][vi] = pkv;
  consumer_sync();
  float kvv = 0.0f;
#pragma unroll
  for (int g = 0; g < NG; ++g) kvv += part[g][vi];
  const float delta = __fmul_rn(__fsub_rn(vs[vi], kvv), ms->gate_beta);
  consumer_sync();
  float po = 0.0f;
#pragma unroll
  for (int kk = 0; kk < KPG; ++kk) {
    const int k = kg * KPG + kk;
    const float s2v = __fadd_rn(sv[kk], __fmul_rn(ks[k], delta));
    Sh[(size_t)k * LV + vi] = s2v;
    po = fmaf(s2v, qs[k], po);
  }
  part[kg][vi] = po;
  consumer_sync();
  if (t < LV) {
    float o = 0.0f;
#pragma unroll
    for (int g = 0; g < NG; ++g) o += part[g][t];
    st_tv(A.tv_o + h * LV + t, o, tag_of(c, p));
  }
  trace_mark(c, p, 2);
  consumer_sync();
  return true;
}

// ---------------------------------------------------------------- attention item

// QK rmsnorm (1+w) + partial RoPE of one 256-vector held by one warp as
// elements lane + 32 q; gains w[] and this lane's cos/sin preloaded.
__device__ __forceinline__ void warp_norm_rope_v(const float* v_in, const float (&w)[8], float co,
                                                 float si, float* dst) {
  const int lane = threadIdx.x & 31;
  float v[8];
  float ss = 0.0f;
#pragma unroll
  for (int q = 0; q < 8; ++q) { v[q] = v_in[lane + 32 * q]; ss = fmaf(v[q], v[q], ss); }
  ss = warp_sum(ss);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), EPS)));
#pragma unroll
  for (int q = 0; q < 8; ++q) v[q] = __fmul_rn(__fmul_rn(v[q], inv), __fadd_rn(1.0f, w[q]));
  const float a = v[0], b = v[1];
  v[0] = __fadd_rn(__fmul_rn(a, co), __fmul_rn(-b, si));
  v[1] = __fadd_rn(__fmul_rn(b, co), __fmul_rn(a, si));
#pragma unroll
  for (int q = 0; q < 8; ++q) dst[lane + 32 * q] = v[q];
}

// Split-KV item (kv group g, chunk cc of nch, positions [cc cl, min(cc cl + cl, T + 1)))
// of attention layer l (golden/model.py:194-229).  The chunk's cached K / V
// rows are read in blocks of ASB = 16 positions, the first block before this
// token's projections can arrive and every next block while the current one
// is used; scores, softmax and P V run as an online (flash-decoding) softmax
// over the blocks: per head a running max m and sum l, and the unnormalised
// output o.  Layouts of a block: K with warp = position, lane = 8 dims; V with
// thread = (dim d, half h) holding positions 8 h .. 8 h + 7.  One chunk
// (nch = 1): o / l * sigmoid(gate) goes straight to tv_attn.  Otherwise the
// chunk's (m, l, o) of its four heads go out as tagged words (att_tv) and
// chunk 0's CTA merges the group: M = max m_c, w_c = exp(m_c - M),
// O = sum w_c o_c / sum w_c l_c, times sigmoid(gate) (golden/model.py:227-229).
// The chunks cover positions [s0, s1) of the Tn = T + 1: all of them, or
// under TP with tp_world > NKV this rank's slice of the group, whose merged
// (m, l, o) chunk 0 then combines with the other slices' (attn_exchange).
constexpr int ASB = 16;
template <bool TP>
__device__ bool attn_exchange(PCtx& c, int p, int hq, int d2, float& M, float& Ls, float& O0, float& O1,
                              unsigned tag);
template <bool TP>
__device__ bool attn_item(PCtx& c, int p, int g, int cc, int nch, int cl, int s0, int s1) {
  const PersistArgs& A = *c.A;
  Misc* ms = c.ms;
  const LayerW& L = c.lay[p / 5];
  const int T = ms->T, pos = ms->pos;
  const int fi = L.full_idx;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int t0 = (TP ? s0 : 0) + cc * cl, t1 = min(TP ? s1 : T + 1, t0 + cl);
  const int tc = min(t1, T);                // positions [t0, tc) come from the cache
  float* qn = (float*)(c.sm + OFF_DIG);    // [4][256] normed + roped queries
  float* kn = qn + 4 * HD;                  // [256] new key
  float* vn = kn + HD;                      // [256] new value
  float* raw = vn + HD;                     // [6][256] projections as read (q x4, k, v)
  float* sp = raw;                          // [2][4][ASB] scores, then probabilities, of alternate blocks (after raw is consumed)
  float* st = sp + 8 * ASB;                 // [4] running max, [4] running sum, [4] rescale
  float* ox = st + 12;                      // [4][256] the second half's o
  const unsigned tin = tag_of(c, p - 1), tout = tag_of(c, p);
  const float* kc = A.kcache + (size_t)fi * A.max_ctx * KVPROJ + g * HD;
  const float* vc = A.vcache + (size_t)fi * A.max_ctx * KVPROJ + g * HD;
  const int d = threadIdx.x & (HD - 1), half = threadIdx.x >> 8;
  // block registers: K (this warp's position, dims 8 lane ..) and V (dim d, 8 positions)
  float kr[8], vr[8];
  auto load_block = [&](int s0) {
    const int tk = s0 + wid;
    if (tk < tc) {
      const float4 a = *reinterpret_cast<const float4*>(kc + (size_t)tk * KVPROJ + 8 * lane);
      const float4 b = *reinterpret_cast<const float4*>(kc + (size_t)tk * KVPROJ + 8 * lane + 4);
      kr[0] = a.x; kr[1] = a.y; kr[2] = a.z; kr[3] = a.w; kr[4] = b.x; kr[5] = b.y; kr[6] = b.z; kr[7] = b.w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int tv = s0 + 8 * half + j;
      vr[j] = tv < tc ? vc[(size_t)tv * KVPROJ + d] : 0.0f;
    }
  };
  load_block(t0);
  // this warp's norm gains and RoPE cos/sin, before waiting
  float nw[8];
  const float* wsrc = (wid < 4) ? L.qn_w : L.kn_w;
#pragma unroll
  for (int q = 0; q < 8; ++q) nw[q] = __ldg(wsrc + lane + 32 * q);
  const float* rope = A.rope + (size_t)pos * ROT;
  const float rco = __ldg(rope + lane), rsi = __ldg(rope + 32 + lane);
  // wait for q (4 heads), k, v of this group (tagged, from IN); element e of
  // [0, 1536): e < 1024 -> q of head 4g + e/256; then k; then v
  {
    const unsigned long long tw = gtime();
    constexpr int NP = (6 * HD / 2 + PT - 1) / PT;   // pairs per thread (2)
    unsigned pend = 0;
#pragma unroll
    for (int jj = 0; jj < NP; ++jj)
      if ((int)threadIdx.x + PT * jj < 6 * HD / 2) pend |= 1u << jj;
    int it = 0;
    for (;;) {
      unsigned long long a[NP], b[NP];
#pragma unroll
      for (int jj = 0; jj < NP; ++jj) {
        if (!(pend >> jj & 1)) continue;
        const int e = 2 * ((int)threadIdx.x + PT * jj);
        const unsigned long long* src;
        if (e < 4 * HD) src = A.tv_qg + (size_t)(4 * g + e / HD) * 2 * HD + (e % HD);
        else if (e < 5 * HD) src = A.tv_kvn + g * HD + (e - 4 * HD);
        else src = A.tv_kvn + KVPROJ + g * HD + (e - 5 * HD);
        ld_tv2(src, a[jj], b[jj]);
      }
#pragma unroll
      for (int jj = 0; jj < NP; ++jj) {
        if ((pend >> jj & 1) && tag_ok(a[jj], tin) && tag_ok(b[jj], tin)) {
          const int e = 2 * ((int)threadIdx.x + PT * jj);
          raw[e] = tv_val(a[jj]);
          raw[e + 1] = tv_val(b[jj]);
          pend &= ~(1u << jj);
        }
      }
      if (consumer_and(pend == 0)) break;
      if (((++it) & 15) == 0) {
        int bad = 0;
        if (threadIdx.x == 0) {
          if (aborted(c)) bad = 1;
          else if (gtime() - tw > WAIT_NS) { raise_abort(c, 19, p); bad = 1; }
        }
        if (!consumer_and(!bad)) return false;
      }
    }
  }
  trace_mark(c, p, 1);
  if (wid < 5) warp_norm_rope_v(raw + wid * HD, nw, rco, rsi, wid < 4 ? qn + wid * HD : kn);   // kn follows qn
  else if (wid == 5) for (int e = lane; e < HD; e += 32) vn[e] = raw[5 * HD + e];
  consumer_sync();
  if (threadIdx.x < 4) { st[threadIdx.x] = -INFINITY; st[4 + threadIdx.x] = 0.0f; }
  if (cc == 0 && threadIdx.x < HD) {   // roped K and raw V into slot T (golden/model.py:216-217)
    A.kcache[((size_t)fi * A.max_ctx + T) * KVPROJ + g * HD + threadIdx.x] = kn[threadIdx.x];
    A.vcache[((size_t)fi * A.max_ctx + T) * KVPROJ + g * HD + threadIdx.x] = vn[threadIdx.x];
  }
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  int par = 0;   // which of the two score buffers this block uses
  for (int s0 = t0; s0 < t1; s0 += ASB, par ^= 1) {
    const int nb = min(ASB, t1 - s0);
    float* spc = sp + par * 4 * ASB;
    // scores of the block (256^-0.5, exact): warp = position
    if (wid < nb) {
      const int tp = s0 + wid;
      float kk[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) kk[i] = tp < T ? kr[i] : kn[8 * lane + i];
#pragma unroll
      for (int hq = 0; hq < 4; ++hq) {
        const float4 q0 = *reinterpret_cast<const float4*>(qn + hq * HD + 8 * lane);
        const float4 q1 = *reinterpret_cast<const float4*>(qn + hq * HD + 8 * lane + 4);
        float dt = q0.x * kk[0] + q0.y * kk[1] + q0.z * kk[2] + q0.w * kk[3];
        dt += q1.x * kk[4] + q1.y * kk[5] + q1.z * kk[6] + q1.w * kk[7];
        dt = warp_sum(dt);
        if (lane == 0) spc[hq * ASB + wid] = dt * 0.0625f;
      }
    }
    // the block's V stays in registers; the next block's K can be requested now
    float vb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) vb[j] = vr[j];
    if (s0 + ASB < t1) load_block(s0 + ASB);
    consumer_sync();
    // online softmax: warp hq < 4 updates head hq
    if (wid < 4) {
      const float sv = lane < nb ? spc[wid * ASB + lane] : -INFINITY;
      const float mold = st[wid];
      const float mnew = fmaxf(mold, warp_max(sv));
      const float pe = lane < nb ? expf(sv - mnew) : 0.0f;
      const float ls = warp_sum(pe);
      if (lane < ASB) spc[wid * ASB + lane] = pe;
      if (lane == 0) {
        const float sc = mold == -INFINITY ? 0.0f : expf(mold - mnew);
        st[8 + wid] = sc;
        st[4 + wid] = fmaf(st[4 + wid], sc, ls);
        st[wid] = mnew;
      }
    }
    consumer_sync();
    // P V over this thread's 8 positions of the block
#pragma unroll
    for (int hq = 0; hq < 4; ++hq) o[hq] = __fmul_rn(o[hq], st[8 + hq]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int tv = s0 + 8 * half + j;
      if (tv < t1) {
        const float vv = tv < T ? vb[j] : vn[d];
#pragma unroll
        for (int hq = 0; hq < 4; ++hq) o[hq] = fmaf(spc[hq * ASB + 8 * half + j], vv, o[hq]);
      }
    }
    // no barrier here: the next block's scores go to the other buffer, and
    // its softmax waits behind a barrier every thread reaches after this P V
  }
  // the two halves' o
  if (half == 1) {
#pragma unroll
    for (int hq = 0; hq < 4; ++hq) ox[hq * HD + d] = o[hq];
  }
  consumer_sync();
  if (half == 0) {
#pragma unroll
    for (int hq = 0; hq < 4; ++hq) o[hq] = __fadd_rn(o[hq], ox[hq * HD + d]);
  }
  // the output gates (in q_proj's [q | gate] rows, written by IN with q): head 4g + hq, dim e
  auto gate = [&](int hq, int e, int& bad) -> float {
    const unsigned long long* gp = A.tv_qg + (size_t)(4 * g + hq) * 2 * HD + HD + e;
    unsigned long long w = ld_tv(gp);
    const unsigned long long tw = gtime();
    int it = 0;
    while (!bad && !tag_ok(w, tin)) {
      if (((++it) & 63) == 0) {
        if (aborted(c)) bad = 1;
        else if (gtime() - tw > WAIT_NS) { raise_abort(c, 20, p); bad = 1; }
      }
      w = ld_tv(gp);
    }
    return tv_val(w);
  };
  int bad = 0;
  const bool xsplit = TP && A.tp_world > NKV;   // the group's positions are split across ranks
  if (nch == 1 && !xsplit) {
    // the whole group in this chunk: o / l * sigmoid(gate)
    if (half == 0) {
#pragma unroll
      for (int hq = 0; hq < 4; ++hq) {
        const float gt = gate(hq, d, bad);
        st_tv(A.tv_attn + (4 * g + hq) * HD + d, __fmul_rn(__fdiv_rn(o[hq], st[4 + hq]), sigmoid_f(gt)), tout);
      }
    }
    trace_mark(c, p, 2);
    return consumer_and(!bad) != 0;
  }
  // this chunk's (m, l, o) of the four heads as tagged words
  unsigned long long* part = A.att_tv + ((size_t)(g * ATT_MAXCH + cc) * 4) * (2 + HD);
  if (half == 0) {
#pragma unroll
    for (int hq = 0; hq < 4; ++hq) {
      st_tv(part + hq * (2 + HD) + 2 + d, o[hq], tout);
      if (d == 0) {
        st_tv(part + hq * (2 + HD), st[hq], tout);
        st_tv(part + hq * (2 + HD) + 1, st[4 + hq], tout);
      }
    }
  }
  trace_mark(c, p, 2);
  if (cc != 0) return consumer_and(1) != 0;
  // chunk 0's CTA merges the group: thread = (head hq, dims 2 d2, 2 d2 + 1),
  // chunks in order (online: running max M, sum Ls, output O)
  const int hq = threadIdx.x >> 7, d2 = 2 * (threadIdx.x & 127);
  const unsigned long long* pb = A.att_tv + ((size_t)(g * ATT_MAXCH) * 4 + hq) * (2 + HD);
  const size_t stride = 4 * (2 + HD);
  float M = -INFINITY, Ls = 0.0f, O0 = 0.0f, O1 = 0.0f;
  for (int q = 0; q < nch && !bad; ++q) {
    const unsigned long long* pq_ = pb + q * stride;
    unsigned long long wm, wl, w0, w1;
    const unsigned long long tw = gtime();
    int it = 0;
    for (;;) {
      wm = ld_tv(pq_);
      wl = ld_tv(pq_ + 1);
      ld_tv2(pq_ + 2 + d2, w0, w1);
      if (tag_ok(wm, tout) && tag_ok(wl, tout) && tag_ok(w0, tout) && tag_ok(w1, tout)) break;
      if (((++it) & 63) == 0) {
        if (aborted(c)) { bad = 1; break; }
        if (gtime() - tw > WAIT_NS) { raise_abort(c, 22, p); bad = 1; break; }
      }
    }
    if (bad) break;
    const float mq = tv_val(wm), lq = tv_val(wl);
    if (mq == -INFINITY) continue;   // an empty slice (TP split with Tn < ranks of the group)
    const float Mn = fmaxf(M, mq);
    const float a = M == -INFINITY ? 0.0f : expf(M - Mn), b = expf(mq - Mn);
    Ls = fmaf(lq, b, __fmul_rn(Ls, a));
    O0 = fmaf(tv_val(w0), b, __fmul_rn(O0, a));
    O1 = fmaf(tv_val(w1), b, __fmul_rn(O1, a));
    M = Mn;
  }
  if constexpr (TP) {
    if (xsplit && !bad && !attn_exchange<TP>(c, p, hq, d2, M, Ls, O0, O1, tout)) bad = 1;
  }
  if (!bad) {
    const float ga = gate(hq, d2, bad), gb = gate(hq, d2 + 1, bad);
    st_tv(A.tv_attn + (4 * g + hq) * HD + d2, __fmul_rn(__fdiv_rn(O0, Ls), sigmoid_f(ga)), tout);
    st_tv(A.tv_attn + (4 * g + hq) * HD + d2 + 1, __fmul_rn(__fdiv_rn(O1, Ls), sigmoid_f(gb)), tout);
  }
  return consumer_and(!bad) != 0;
}

// The attention sequence split (TP, tp_world > NKV): the ns = tp_world / NKV
// ranks of a KV group each hold the merged (m, l, o) of their position slice
// (thread = head hq, dims d2, d2 + 1).  Each stores it as tagged words into
// slot j = tp_rank % ns of every group rank's exchange buffer (NVLink P2P,
// system scope), then merges slots 0 .. ns-1 in order, skipping empty slices
// (m = -inf): the same combine as the chunks' (golden/model.py:219-229), in an
// order every rank of the group shares, so their outputs are bit-identical.
// A slot is rewritten four layers later, after the OUT and DOWN exchanges in
// between have shown that every rank has read it.
template <bool TP>
__device__ bool attn_exchange(PCtx& c, int p, int hq, int d2, float& M, float& Ls, float& O0, float& O1,
                              unsigned tag) {
  const PersistArgs& A = *c.A;
  const int ns = A.tp_world / NKV, j = A.tp_rank % ns, r0 = A.tp_rank - j;
  constexpr size_t SW = 2 + HD;   // words per head
  const size_t mine = XB_ATT + ((size_t)j * 4 + hq) * SW;
  for (int q = 0; q < ns; ++q) {
    unsigned long long* dst = A.xbuf[r0 + q] + mine;
    st_tv_sys(dst + 2 + d2, O0, tag);
    st_tv_sys(dst + 3 + d2, O1, tag);
    if (d2 == 0) {
      st_tv_sys(dst, M, tag);
      st_tv_sys(dst + 1, Ls, tag);
    }
  }
  const unsigned long long* xb = A.xbuf[A.tp_rank] + XB_ATT + (size_t)hq * SW;
  float m2 = -INFINITY, l2 = 0.0f, p0 = 0.0f, p1 = 0.0f;
  for (int q = 0; q < ns; ++q) {
    const unsigned long long* src = xb + (size_t)q * 4 * SW;
    unsigned long long wm, wl, w0, w1;
    const unsigned long long tw = gtime();
    int it = 0;
    for (;;) {
      wm = ld_tv_sys(src);
      wl = ld_tv_sys(src + 1);
      w0 = ld_tv_sys(src + 2 + d2);
      w1 = ld_tv_sys(src + 3 + d2);
      if (tag_ok(wm, tag) && tag_ok(wl, tag) && tag_ok(w0, tag) && tag_ok(w1, tag)) break;
      if (((++it) & 63) == 0) {
        if (aborted(c)) return false;
        if (gtime() - tw > WAIT_NS) { raise_abort(c, 23, p | q << 8); return false; }
      }
    }
    const float mq = tv_val(wm);
    if (mq == -INFINITY) continue;
    const float Mn = fmaxf(m2, mq);
    const float a = m2 == -INFINITY ? 0.0f : expf(m2 - Mn), b = expf(mq - Mn);
    l2 = fmaf(tv_val(wl), b, __fmul_rn(l2, a));
    p0 = fmaf(tv_val(w0), b, __fmul_rn(p0, a));
    p1 = fmaf(tv_val(w1), b, __fmul_rn(p1, a));
    m2 = Mn;
  }
  M = m2;
  Ls = l2;
  O0 = p0;
  O1 = p1;
  return true;
}

// ---------------------------------------------------------------- the kernel

// TP: the tensor-parallel instances (launched when tp_world > 1); the others
// compile every exchange out.  I8: the ACT_INT8 (W8A8) instances; the W8A32
// ones compile the int8 activation quantisers out of their GEMV phases.
template <bool TP, bool I8>
__global__ void __launch_bounds__(NTHREADS, 1) k_decode_persistent(PersistArgs A) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw;
  PCtx c;
  c.A = &A;
  c.sm = sm;
  c.ms = (Misc*)(sm + OFF_MISC);
  c.lay = (LayerW*)(sm + OFF_LAY);
  Chunk* chs = (Chunk*)(sm + OFF_CH);
  c.ch = chs;
  c.nch = A.phase_first[(size_t)blockIdx.x * (NPHASE + 1) + NPHASE];
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(c.pol));
  const unsigned long long t_entry = gtime();
  Misc* ms = c.ms;
  // stage the layer table, this CTA's chunk list and the step scalars
  for (int i = threadIdx.x; i < (int)(sizeof(LayerW) * NLAYER / 4); i += NTHREADS)
    ((int*)c.lay)[i] = ((const int*)A.layers)[i];
  for (int i = threadIdx.x; i < c.nch; i += NTHREADS) chs[i] = A.chunks[(size_t)blockIdx.x * MAXCH + i];
  for (int i = threadIdx.x; i <= NPHASE; i += NTHREADS) ms->pf[i] = A.phase_first[(size_t)blockIdx.x * (NPHASE + 1) + i];
  for (int i = threadIdx.x; i < MAXPAN * 4 * PANEL; i += NTHREADS) ((int*)(sm + OFF_PART))[i] = 0;
  if (threadIdx.x < 2 * NCW) ms->rfq[threadIdx.x >> 1][threadIdx.x & 1] = 0;
  if (threadIdx.x == 0) {
    ms->amax[0] = 0u;
    ms->amax[1] = 0u;
    ms->abort = 0;
    ms->pos = A.dyn->pos;
    ms->T = A.dyn->T;
    ms->conv_base = A.dyn->conv_base;
    ms->act_int8 = A.dyn->act_int8;
    ms->want_logits = A.dyn->want_logits;
    ms->seq = A.dyn->seq;
    const int step = A.io[0], np = A.io[1];
    ms->step = step;
    int tok = (step < np) ? A.io[2 + step] : A.ids[step > 0 ? step - 1 : 0];
    if (tok < 0 || tok >= VOCAB) { atomicCAS(A.err, 0, ERR_TOKEN); tok = 0; }
    ms->tok = tok;
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(full_bar(c, s), 1);
      mbar_init(mma_bar(c, s), 1);
      ms->slot_last[s] = -1;
    ms->pcnt[s] = 0;
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf_bar(c, b), 1);
      mbar_init(acce_bar(c, b), 4);
    }
    mbar_init(fin_bar(c), 1);
    ms->ntile = 0;
    ms->mpar = 0;
    ms->mma_any = 0;
    ms->hs_tag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (ms->T >= A.max_ctx || ms->pos >= A.max_rope) {
    if (threadIdx.x == 0) atomicCAS(A.err, 0, ERR_CTX);
    return;
  }
  // 32 TMEM columns: the head's two 128 x 16 int32 accumulators.  One CTA per
  // SM (the launch holds the whole register file), so the allocation is free.
  if ((threadIdx.x >> 5) == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 32;"
                 :: "r"(smem_u32(&ms->tmem)) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (A.trace && threadIdx.x == 0) {   // kernel entry and TMEM ready, in the unused stamps of phase 1
    A.trace[((size_t)blockIdx.x * NPHASE + 1) * TRACE_STAMPS + 1] = t_entry;
    A.trace[((size_t)blockIdx.x * NPHASE + 1) * TRACE_STAMPS + 2] = gtime();
  }
  if (threadIdx.x == 0)
    for (int i = 0; i < NSLOT && i < c.nch; ++i) {
      issue_chunk(c, i);
      ms->slot_last[i] = i;
    }
  {
    bool ok = true;
    for (int p = 0; p < NPHASE && ok; ++p) {
      const int sub = p % 5;
      trace_mark(c, p, 0);
      if (ms->rfq[threadIdx.x >> 5][0]) do_refills(c);   // the slots this warp's finished panels released
      if (p != PH_HEAD && sub == 1) {
        const LayerW& L = c.lay[p / 5];
        if (L.linear) {
          // this rank's heads [dn_h0, dn_h1): CTA j runs head dn_h0 + j
          const int h0 = TP ? A.dn_h0 : 0, nh = TP ? A.dn_h1 - A.dn_h0 : LH;
          if ((int)blockIdx.x < nh) ok = delta_head(c, p, h0 + blockIdx.x);
        } else {
          // chunks of ASB positions (at most ATT_MAXCH, and one item per CTA)
          const int g0 = TP ? A.kv_g0 : 0, ng = TP ? A.kv_g1 - A.kv_g0 : NKV;   // this rank's KV groups
          const int Tn = ms->T + 1;
          int s0 = 0, s1 = Tn;   // positions of this rank (TP, tp_world > NKV: its slice of the group)
          if (TP && A.tp_world > NKV) {
            const int ns = A.tp_world / NKV, j = A.tp_rank % ns;
            s0 = j * Tn / ns;
            s1 = (j + 1) * Tn / ns;
          }
          int nch = (s1 - s0 + ASB - 1) / ASB;
          const int cap = min(ATT_MAXCH, (int)gridDim.x / ng);
          nch = nch < 1 ? 1 : (nch > cap ? cap : nch);
          const int cl = (s1 - s0 + nch - 1) / nch;
          for (int it = blockIdx.x; it < ng * nch && ok; it += gridDim.x)
            ok = attn_item<TP>(c, p, g0 + it % ng, it / ng, nch, cl, s0, s1);
        }
        trace_mark(c, p, 3);
        continue;
      }
      // this phase's chunks, [i0, i1) of the CTA's list (counted loops only)
      const int i0 = ms->pf[p], i1 = ms->pf[p + 1];
      const int nhead = TP ? A.dn_h1 - A.dn_h0 : LH;
      if (p != PH_HEAD && sub == 0 && c.lay[p / 5].linear && (int)blockIdx.x < nhead) {
        // a DeltaNet head's CTA: the head's gate inputs (it holds no panels)
        ok = consumer_and(gate_inputs(c, p, (TP ? A.dn_h0 : 0) + blockIdx.x)) != 0;
        trace_mark(c, p, 3);
        continue;
      }
      if (p == PH_HEAD) {
        ok = phase_head<TP>(c, p, i0, i1);       // every CTA joins the argmax merge
      } else if (i0 == i1) {                     // no rows of this phase on this CTA
        trace_mark(c, p, 3);
        continue;
      } else {
        ok = (sub == 0 || sub == 3) ? phase_panels<TP, I8, true>(c, p, i0, i1)
                                     : phase_panels<TP, I8, false>(c, p, i0, i1);
      }
      // the warps leave a GEMV phase independently; line them up again (and
      // make a failure in any warp the whole CTA's)
      ok = consumer_and(ok) != 0;
      trace_mark(c, p, 3);
    }
    if (!ok && threadIdx.x == 0) *(volatile int*)&ms->abort = 1;
  }
  // every MMA the CTA issued has completed before its shared memory and tensor
  // memory are released (on an abort path nobody else waited for them)
  if (threadIdx.x == (NCW - 1) * 32 && ms->mma_any) {
    umma_commit(fin_bar(c));
    const unsigned long long t0 = gtime();
    while (!mbar_try(fin_bar(c), 0u))
      if (gtime() - t0 > WAIT_NS) { atomicCAS(A.err, 0, ERR_WAIT); break; }
  }
  // drain: every bulk copy that was issued must land before the CTA exits
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long t0 = gtime();
    for (int s = 0; s < NSLOT; ++s) {
      const int last = ms->slot_last[s];
      if (last < 0) continue;
      const unsigned bar = full_bar(c, s);
      while (!mbar_try(bar, (unsigned)((last / NSLOT) & 1)))
        if (gtime() - t0 > WAIT_NS) break;
    }
  }
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" :: "r"(ms->tmem) : "memory");
  }
}

static_assert(OFF_DIG + (4 * HD + 2 * HD + 6 * HD) * 4 <= OFF_HS && 8 * ASB + 12 + 4 * HD <= 6 * HD,
              "attention scratch must fit in the digit/xf region");

}  // namespace

// ---------------------------------------------------------------- host side
//
// persist_tp.cu compiles this file a second time with QB_PERSIST_TP defined:
// that translation unit holds only the tensor-parallel kernel instance and its
// launcher, so the single-GPU kernel's code here is laid out without any of
// the exchange paths (measured: 8 us per step when both shared one module).

// Launch one instance (cooperative: every CTA resident, one per SM).
template <bool TP, bool I8>
cudaError_t launch_instance(const PersistArgs& args, int G, cudaStream_t st) {
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k_decode_persistent<TP, I8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  void* kargs[] = {(void*)&args};
  return cudaLaunchCooperativeKernel((const void*)k_decode_persistent<TP, I8>, dim3(G), dim3(NTHREADS), kargs,
                                     SMEM_BYTES, st);
}
// Resident CTAs per SM of the smaller of an instance pair.
template <bool TP>
int blocks_per_sm() {
  int n0 = 0, n1 = 0;
  cudaFuncSetAttribute(k_decode_persistent<TP, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  cudaFuncSetAttribute(k_decode_persistent<TP, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n0, k_decode_persistent<TP, false>, NTHREADS, SMEM_BYTES);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n1, k_decode_persistent<TP, true>, NTHREADS, SMEM_BYTES);
  return n0 < n1 ? n0 : n1;
}

#ifdef QB_PERSIST_TP
cudaError_t launch_persistent_tp(const PersistArgs& args, int G, cudaStream_t st, bool i8) {
  return i8 ? launch_instance<true, true>(args, G, st) : launch_instance<true, false>(args, G, st);
}
int persist_tp_max_blocks_per_sm() { return blocks_per_sm<true>(); }
#else
cudaError_t launch_persistent_tp(const PersistArgs& args, int G, cudaStream_t st, bool i8);   // persist_tp.cu
int persist_tp_max_blocks_per_sm();

int persist_smem_bytes() { return SMEM_BYTES; }
int persist_num_phases() { return NPHASE; }
int persist_max_chunks() { return MAXCH; }
size_t persist_trace_words(int G) {
  return (size_t)G * NPHASE * TRACE_STAMPS + (size_t)NPHASE * NCW * TRACE_WARP_STAMPS;
}


// Build the per-CTA chunk lists.
//   IN, OUT, GATEUP, DOWN: whole panels (16 rows, GATEUP 8 gate + 8 up; all of a panel's K-slices on
//     one CTA).  Each panel goes to the CTA with the fewest 4 KB tasks so far
//     in the phase, then the fewest bytes so far in the step, then the lowest
//     index, among the CTAs whose ring still holds the panel's chunks with the
//     phase's others.  The first nh CTAs (nh = the rank's DeltaNet heads) hold
//     no panels: CTA j runs DeltaNet head dn_h0 + j (gate inputs in IN, the
//     delta rule in MIX).
//   HEAD: contiguous, balanced ranges of the 1940 tiles over every CTA.
bool tp_plan(int rank, int world, TpPlan& out, std::string& err) {
  if (world != 1 && world != 2 && world != 4 && world != TP_MAX) { err = "tp world must be 1, 2, 4 or 8"; return false; }
  if (rank < 0 || rank >= world) { err = "tp rank outside [0, world)"; return false; }
  TpPlan t;
  t.rank = rank;
  t.world = world;
  t.dn_h0 = LH * rank / world;
  t.dn_h1 = LH * (rank + 1) / world;
  if (world <= NKV) {
    t.kv_g0 = NKV * rank / world;
    t.kv_g1 = NKV * (rank + 1) / world;
  } else {   // the KV group of this rank's query heads (computed by world / NKV ranks)
    t.kv_g0 = (NH * rank / world) / (NH / NKV);
    t.kv_g1 = t.kv_g0 + 1;
  }
  t.ok0 = VDIM * rank / world;   // = the rank's DeltaNet heads x LV = its query heads x HD
  t.ok1 = VDIM * (rank + 1) / world;
  constexpr int NB = FFN / 128;  // FFN columns in blocks of 128 (whole MMA task pieces)
  t.dk0 = 128 * (NB * rank / world);
  t.dk1 = 128 * (NB * (rank + 1) / world);
  t.t0 = (int)((long long)HEAD_TILES * rank / world);
  t.t1 = (int)((long long)HEAD_TILES * (rank + 1) / world);
  out = t;
  return true;
}

bool build_schedule(const ModelW& M, int G, const TpPlan& tp, std::vector<Chunk>& chunks,
                    std::vector<unsigned short>& phase_first, std::string& err) {
  (void)M;
  if (G < 1) { err = "no CTAs"; return false; }
  chunks.assign((size_t)G * MAXCH, Chunk{});
  phase_first.assign((size_t)G * (NPHASE + 1), 0);
  std::vector<int> counts(G, 0);
  std::vector<long long> load(G, 0);
  auto push = [&](int b, int p, int seg, int n, int row0, int bytes) -> bool {
    int& cnt = counts[b];
    if (cnt >= MAXCH) { err = "chunk list overflow"; return false; }
    Chunk& k = chunks[(size_t)b * MAXCH + cnt++];
    k.phase = (unsigned short)p;
    k.seg = (unsigned char)seg;
    k.nrows = (unsigned char)n;
    k.row0 = (unsigned)row0;
    load[b] += bytes;
    return true;
  };
  // Time model of the step (us, from traces of this kernel): an idle CTA sees
  // a phase's input T_PROP after the last producer wrote it; a CTA that worked
  // in a phase is free again T_REL after its outputs (slot refills, phase
  // exit, the next phase's set-up); a GEMV phase costs T_ENC + T_ROUND per
  // round of NCW tasks + T_TAIL from its start; the DeltaNet / attention MIX
  // items take T_DELTA / T_ATTN.  Panels go to the CTA that would finish the
  // phase earliest, so a phase's work avoids the CTAs still busy with the last.
  constexpr double T_PROP = 0.6, T_REL = 1.8, T_ENC = 0.5, T_TAIL = 0.45;
  constexpr double T_ROUND = 0.2 + 0.5 * TASK_KB / 512.0;   // one task per warp
  constexpr double T_DELTA = 2.4, T_ATTN = 4.0;
  constexpr int ATT_CTAS = 20;   // CTAs running attention items at short contexts
  const int nhead = tp.dn_h1 - tp.dn_h0;   // CTAs [0, nhead): the DeltaNet heads, no panels
  if (G <= nhead) { err = "fewer CTAs than DeltaNet heads"; return false; }
  std::vector<double> freeb(G, 0.0);
  double ready = 0.0;            // when the current phase's input reaches an idle CTA
  for (int p = 0; p < NPHASE; ++p) {
    // every CTA's chunks of phase p start where its list stands now
    for (int b = 0; b < G; ++b) phase_first[(size_t)b * (NPHASE + 1) + p] = (unsigned short)counts[b];
    const int sub = p % 5;
    if (p == PH_HEAD) {
      // whole tiles per CTA (a tile's K-slabs accumulate in one CTA's TMEM)
      const int nt = tp.t1 - tp.t0;   // this rank's vocab slice
      for (int b = 0; b < G; ++b) {
        const int t0 = tp.t0 + (int)((long long)nt * b / G), t1 = tp.t0 + (int)((long long)nt * (b + 1) / G);
        for (int t = t0; t < t1; ++t)
          for (int j = 0; j < HEAD_NSLAB; ++j)
            if (!push(b, p, CHUNK_MMA, j, t, SLOTW)) return false;
      }
      continue;
    }
    const bool linear = (p / 5) % 4 != 3;
    if (sub == 1) {
      double last = ready;
      for (int b = 0; b < G; ++b)
        if (linear ? b < nhead : b < ATT_CTAS) {
          freeb[b] = std::max(freeb[b], ready) + (linear ? T_DELTA : T_ATTN);
          last = std::max(last, freeb[b]);
        }
      ready = last + T_PROP;
      continue;
    }
    // this rank's panels of the phase and its K window
    std::vector<int> pans;
    int kw0 = 0, kw1 = HID;
    if (sub == 0) {
      if (linear) {   // q, k, v, z blocks of 2048 rows; head h = 8 panels of each
        for (int blk = 0; blk < 4; ++blk)
          for (int h = tp.dn_h0; h < tp.dn_h1; ++h)
            for (int j = 0; j < LK / PANEL; ++j) pans.push_back(blk * (KDIM / PANEL) + h * (LK / PANEL) + j);
      } else {        // the KV groups' query heads ([q | gate] rows), then their k rows, then v rows
        for (int g = tp.kv_g0; g < tp.kv_g1; ++g)
          for (int j = 0; j < QPROJ / NKV / PANEL; ++j) pans.push_back(g * (QPROJ / NKV / PANEL) + j);
        for (int kv = 0; kv < 2; ++kv)
          for (int g = tp.kv_g0; g < tp.kv_g1; ++g)
            for (int j = 0; j < HD / PANEL; ++j) pans.push_back((QPROJ + kv * KVPROJ + g * HD) / PANEL + j);
      }
    } else if (sub == 3) {
      for (int q = tp.dk0 / PAIR_ROWS; q < tp.dk1 / PAIR_ROWS; ++q) pans.push_back(q);
    } else {
      for (int q = 0; q < HID / PANEL; ++q) pans.push_back(q);
      kw0 = sub == 2 ? tp.ok0 : tp.dk0;
      kw1 = sub == 2 ? tp.ok1 : tp.dk1;
    }
    // a panel's K-slices of the window: bytes and tasks of each
    std::vector<int> sl_bytes, sl_tasks;
    for (int k0 = kw0; k0 < kw1; k0 += PANEL_KB) {
      const int kb = kw1 - k0 < PANEL_KB ? kw1 - k0 : PANEL_KB;
      sl_bytes.push_back(PANEL * kb);
      sl_tasks.push_back((kb + TASK_KB - 1) / TASK_KB);
    }
    const int nslice = (int)sl_bytes.size();
    int ptasks = 0;
    for (int x : sl_tasks) ptasks += x;
    std::vector<int> inph(G, 0), tasks(G, 0);   // chunks (at most NSLOT: all resident at once) and tasks
    auto fin_of = [&](int b, int t) {
      return std::max(freeb[b], ready) + T_ENC + T_ROUND * ((t + NCW - 1) / NCW) + T_TAIL;
    };
    auto least_fit = [&](int need, int add) {
      int best = -1;
      double fb = 0.0;
      for (int b = nhead; b < G; ++b) {
        if (inph[b] + need > NSLOT) continue;
        const double f = fin_of(b, tasks[b] + add);
        if (best < 0 || f < fb - 1e-9 ||
            (f < fb + 1e-9 && (tasks[b] < tasks[best] || (tasks[b] == tasks[best] && load[b] < load[best])))) {
          best = b;
          fb = f;
        }
      }
      return best;
    };
    for (int q : pans) {
      const int b = least_fit(nslice, ptasks);
      if (b < 0) { err = "phase does not fit the rings"; return false; }
      inph[b] += nslice;
      tasks[b] += ptasks;
      for (int j = 0; j < nslice; ++j)
        if (!push(b, p, CHUNK_PANEL, j, q, sl_bytes[j])) return false;
    }
    double last = ready;
    for (int b = 0; b < G; ++b)
      if (tasks[b]) {
        const double f = fin_of(b, tasks[b]);
        freeb[b] = f + T_REL;
        last = std::max(last, f);
      }
    ready = last + T_PROP;
  }
  for (int b = 0; b < G; ++b) phase_first[(size_t)b * (NPHASE + 1) + NPHASE] = (unsigned short)counts[b];
  return true;
}

// One 16-byte core-matrix row per thread: tile t, slab j, row m, K-group g.
__global__ void k_repack_head(const int4* __restrict__ emb, int4* __restrict__ tiles) {
  const size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  constexpr int G16 = HEAD_KS / 16;
  if (id >= (size_t)VOCAB * (HID / 16)) return;
  const int g = (int)(id % G16);
  const int m = (int)((id / G16) % HEAD_TM);
  const int j = (int)((id / (G16 * HEAD_TM)) % HEAD_NSLAB);
  const size_t t = id / ((size_t)G16 * HEAD_TM * HEAD_NSLAB);
  const int4 v = emb[((t * HEAD_TM + m) * HID + (size_t)j * HEAD_KS) / 16 + g];
  tiles[((t * HEAD_NSLAB + j) * (HEAD_TM * HEAD_KS) + ((m >> 3) * G16 + g) * 128 + (m & 7) * 16) / 16] = v;
}

cudaError_t repack_head_tiles(const int8_t* emb_q, int8_t* tiles, cudaStream_t st) {
  if (((uintptr_t)emb_q & 15) || ((uintptr_t)tiles & 15)) return cudaErrorMisalignedAddress;
  const size_t n = (size_t)VOCAB * (HID / 16);
  k_repack_head<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(reinterpret_cast<const int4*>(emb_q),
                                                          reinterpret_cast<int4*>(tiles));
  return cudaGetLastError();
}

// Re-lay rows as 16-row panels: thread = one 16-byte K-group of one row.
__global__ void k_repack_panels(const int8_t* const* __restrict__ rowptr, int4* __restrict__ out, int nrows,
                                int K) {
  const size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int G16 = K / 16;
  if (id >= (size_t)nrows * G16) return;
  const int g = (int)(id % G16);
  const size_t r = id / G16;
  const int4 v = reinterpret_cast<const int4*>(rowptr[r])[g];
  const size_t q = r / PANEL;
  const int m = (int)(r % PANEL);
  out[(q * PANEL * K + ((size_t)g * PANEL + m) * 16) / 16] = v;
}

cudaError_t repack_panels(const int8_t* const* rowptr, int8_t* out, int nrows, int K, cudaStream_t st) {
  if (nrows % PANEL || K % TASK_KB || ((uintptr_t)out & 15)) return cudaErrorInvalidValue;
  const size_t n = (size_t)nrows * (K / 16);
  k_repack_panels<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rowptr, reinterpret_cast<int4*>(out), nrows, K);
  return cudaGetLastError();
}

cudaError_t launch_persistent(const PersistArgs& args, int G, cudaStream_t st, bool i8) {
  if (args.tp_world > 1) return launch_persistent_tp(args, G, st, i8);
  return i8 ? launch_instance<false, true>(args, G, st) : launch_instance<false, false>(args, G, st);
}

// Resident CTAs per SM of the persistent kernel (the smallest of its instances).
int persist_max_blocks_per_sm() {
  const int n = blocks_per_sm<false>();
  const int n1 = persist_tp_max_blocks_per_sm();
  return n < n1 ? n : n1;
}
#endif  // QB_PERSIST_TP

}  // namespace qb
