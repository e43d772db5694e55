// worker.cuh — the persistent worker (one CTA per SM).
//
// Reference: src/persistent_kernel.cu:138-231.  There, thread 0 of each CTA CAS-claims
// one 496-byte Task, the whole CTA runs it, and completion is a system atomic on a
// mapped counter.  Here:
//   * warp 0 is the dequeue warp: it takes item tickets from a device counter, reads
//     the 64-byte item from the ring in mapped pinned memory, waits on the item's
//     dependency barrier, and stages contiguous operands into shared memory with TMA
//     bulk copies (mbarrier complete_tx), up to `stages` items ahead;
//   * warps 2.. are compute warps: they run the tile function for the item through the
//     device function-pointer table (one indirect call per tile), or, for a reference
//     Task, resolve g_op_alias/g_op_table at dequeue time and run it with the whole CTA;
//     each compute warp signals a per-stage `done` barrier, with no CTA-wide barrier
//     between tiles;
//   * warp 1 is the completer: it returns finished stages to the dequeue warp at once and
//     batches completion accounting (one fence for several items); completion is counted
//     per flush and the last item of a flush writes that flush's ticket into mapped
//     memory (single writer, no host-memory atomics);
//   * every wait is bounded by %globaltimer; a wait that runs out records an error in the
//     mapped report and the grid exits;
//   * exit is coordinated so no ticket is lost: the CTAs park, the leader (CTA 0)
//     publishes EXITING, re-reads the host tail (Dekker-style with the host's publish) and
//     either resumes or lets the grid exit with the exact drain point recorded for the
//     next launch.
#pragma once
#include "tiles.cuh"

namespace gpuos {

constexpr uint64_t kNoTicket = ~0ull;
constexpr uint32_t kBarTask = 2;                            // named barrier: whole CTA

struct WorkerShared {
  SmemHeader* H;
  unsigned char* bufs;
  uint32_t stage_bytes;
  uint64_t load_policy;  // L2 cache policy of operand bulk loads (0: none)
};

__device__ __forceinline__ unsigned char* stage_buf(const WorkerShared& W, uint32_t s) {
  return W.bufs + (size_t)s * W.stage_bytes;
}

__device__ __forceinline__ void report_error(const WorkerParams& P, uint32_t code, uint64_t item,
                                             uint64_t waited_ns = 0, uint64_t bound_ns = 0) {
  if (atomicCAS(&P.dc->abort, 0u, 1u) == 0u) {
    if (bound_ns) P.dc->err_wait = ((waited_ns / 1000) << 32) | (bound_ns / 1000000);
    ptx::st_relaxed_sys(&P.rep->error_item, item);
    ptx::fence_acq_rel_sys();
    ptx::st_relaxed_sys(&P.rep->error, ((uint64_t)code << 32) | (uint32_t)blockIdx.x);
    if (P.sticky_error) atomicCAS(P.sticky_error, 0ull, ((unsigned long long)code << 32) | (uint32_t)blockIdx.x);
  }
}

// First occurrence of a launch event (see TimelineSlot); callers mark each event once.
__device__ __forceinline__ void tl_mark(const WorkerParams& P, int slot) {
  if (gridDim.x < kDiagCtas) atomicMin(&P.dc->diag[gridDim.x][slot], (unsigned long long)ptx::now_ns());
}

// Table lookup at dequeue time (persistent_kernel.cu:184-193).
__device__ __forceinline__ OpFn resolve_op(const WorkerParams& P, int op) {
  if (op < 0 || op >= GPUOS_MAX_OPS) return nullptr;
  const int phys = *reinterpret_cast<volatile int*>(&P.op_alias[op]);
  if (phys < 0 || phys >= GPUOS_MAX_OPS) return nullptr;
  return reinterpret_cast<OpFn>(*reinterpret_cast<volatile unsigned long long*>(&P.op_table[phys]));
}

// ---- completion ----------------------------------------------------------------------
// Completed items of one flush awaiting accounting (the completer warp batches them).
struct DoneRun {
  uint32_t batch, batch_items, batch_seq, n;
};
constexpr int kMaxRuns = 4;
constexpr uint32_t kAccountEvery = 8;  // items per fence when completions stream in

// A flush is complete: its ticket goes out first (the host waits on it), its time stamps
// after.  The system-scope fence before the ticket orders every item of the flush (this
// CTA's stores, and the other CTAs' through the per-flush counter read before it) and the
// slot resets; `tseq` marks the stamps of that flush as written.
__device__ __forceinline__ void finish_flush(const WorkerParams& P, const DoneRun& d) {
  const unsigned long long t_end = ptx::now_ns();
  const unsigned long long t0 = atomicExch(&P.dc->batch_t0[d.batch], ~0ull);
  Ticket& tk = P.tickets[d.batch];
  ptx::fence_acq_rel_sys();
  ptx::st_relaxed_sys(&tk.seq, d.batch_seq);
  ptx::st_relaxed_sys(&tk.t_start, t0);
  ptx::st_relaxed_sys(&tk.t_end, t_end);
  ptx::fence_acq_rel_sys();
  ptx::st_relaxed_sys(&tk.tseq, d.batch_seq);
}

// One gpu-scope fence covers every item of the runs (their compute warps' stores were
// ordered before the completer by the per-stage done barriers); then the per-flush
// counters; the last item of a flush writes the flush's ticket into mapped memory.  A run
// that holds every item of its flush is complete without the counter.
__device__ void account(const WorkerParams& P, const DoneRun* runs, int nruns, bool* first) {
  if (*first) {
    tl_mark(P, TL_ACCOUNT);
    *first = false;
  }
  // a single whole flush needs no gpu-scope release of its own: finish_flush fences at
  // system scope before anything else is written
  if (nruns != 1 || runs[0].n != runs[0].batch_items) ptx::fence_acq_rel_gpu();
  unsigned long long total = 0;
  for (int r = 0; r < nruns; ++r) {
    const DoneRun& d = runs[r];
    total += d.n;
    if (d.n == d.batch_items) {
      finish_flush(P, d);
      continue;
    }
    const unsigned int prev = atomicAdd(&P.dc->batch_done[d.batch], d.n);
    if (prev + d.n == d.batch_items) {
      P.dc->batch_done[d.batch] = 0u;
      finish_flush(P, d);
    }
  }
  atomicAdd(&P.dc->items_done, total);
}

// Bounded wait on an mbarrier phase (one lane).  `alive` is a %globaltimer stamp another
// role refreshes while it makes progress; the wait fails once it is older than `limit`.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, const unsigned long long* alive,
                                           uint64_t limit, uint64_t* waited) {
  uint32_t spins = 0;
  while (!ptx::mbar_try_wait(bar, parity)) {
    if ((++spins & 1023u) == 0) {
      const uint64_t a = *reinterpret_cast<const volatile unsigned long long*>(alive);
      const uint64_t w = ptx::elapsed(ptx::now_ns(), a);
      if (w > limit) {
        *waited = w;
        return false;
      }
    }
  }
  return true;
}

// ---- compute warps ----------------------------------------------------------------------
// Diagnostics of the compute warps (thread 0): cycles waiting for filled stages and inside tiles.
__device__ __forceinline__ void compute_diag(const WorkerParams& P, uint32_t ctid, unsigned long long wait_c,
                                             unsigned long long tile_c, unsigned long long fill_c) {
  if (ctid == 0 && blockIdx.x < kDiagCtas) {
    unsigned long long* row = P.dc->diag[blockIdx.x];
    row[DG_C_WAIT_FULL] = wait_c;
    row[DG_C_TILE] = tile_c;
    row[DG_C_FILL] = fill_c;
  }
}

// ---- runs of table-dispatched tiles ----------------------------------------------------
// A tile reached through a function table is a call, and every call saves and restores the
// callee-saved registers of all compute threads through local memory.  The table therefore
// holds run functions: one call processes the stage it was made for and every following stage
// whose item belongs to the same run function, so the call is paid once per run of items (the
// consecutive tickets of one request that this CTA claimed as a chunk) instead of once per
// item.  A run returns with the full phase of the next stage complete (kRunNext), or after a
// wait that expired, the error reported (kRunError).
struct RunState {
  const WorkerParams* P;
  SmemHeader* H;
  unsigned char* bufs;
  uint32_t stage_bytes, S;
  uint32_t s, parity;  // stage and phase parity of use `iter`
  uint64_t iter;
  uint32_t tid, nt;
  int status;
};
constexpr int kRunNext = 0, kRunError = 1;

// The run function of an item (its index in g_run_fns), one per tile kind and op so that each
// holds a single tile body (with several bodies inlined side by side the register allocation
// spills): [0, N) contiguous tiles of op k, N the generic reductions and top-k, N + 1 + k staged
// transpose blocks of op k, 2N + 1 + k 2-D blocks, 3N + 1 the generic stride walk, 3N + 2 staged
// transpose blocks of the ops of kSharedOps (one shared body, the op switched per quad of
// values: per-op bodies missed in the instruction cache when consecutive blocks changed op); -1
// for the items the compute loop runs itself (N = GPUOS_EW_NUM_OPS).
constexpr int kRunT2d = GPUOS_EW_NUM_OPS + 1, kRun2d = 2 * GPUOS_EW_NUM_OPS + 1,
              kRunGeneric = 3 * GPUOS_EW_NUM_OPS + 1, kRunT2dShared = 3 * GPUOS_EW_NUM_OPS + 2;
__device__ __forceinline__ int run_index(const StageMeta& m) {
  const uint8_t kind = m.item.kind;
  const int op = (int)m.item.op;
  if (kind == IK_EW_CONTIG) return f32_inline_ok(m) ? -1 : op;
  if (kind == IK_EW_2DT) return op < 32 && ((kSharedOps >> op) & 1u) ? kRunT2dShared : kRunT2d + op;
  if (kind == IK_EW_2D) return kRun2d + op;
  if (kind == IK_EW_GENERIC) return kRunGeneric;
  if (kind == IK_RED_GENERIC || kind == IK_TOPK) return GPUOS_EW_NUM_OPS;
  return -1;
}

// Ends the tile of stage s (this warp's done arrival), moves to the next stage and waits for
// it to fill; true when its item belongs to run `idx` too.
__device__ __forceinline__ bool run_advance(RunState& r, uint32_t& s, uint32_t& parity, uint64_t& iter, int idx) {
  SmemHeader& H = *r.H;
  __syncwarp();
  if ((r.tid & 31) == 0) ptx::mbar_arrive(ptx::smem_addr(&H.done[s]));
  ++iter;
  s = s + 1 == r.S ? 0 : s + 1;
  if (s == 0) parity ^= 1u;
  uint64_t waited = 0;
  if (!wait_phase(ptx::smem_addr(&H.full[s]), parity, &H.prod_alive, H.full_wait_ns, &waited)) {
    report_error(*r.P, DE_WAIT_FULL, iter, waited, H.full_wait_ns);
    r.status = kRunError;
    return false;
  }
  r.status = kRunNext;
  return run_index(H.meta[s]) == idx;
}

__device__ __forceinline__ TileCtx run_ctx(const RunState& r, uint32_t s) {
  TileCtx c;
  c.m = &r.H->meta[s];
  c.sa = r.bufs + (size_t)s * r.stage_bytes;
  c.sb = c.sa + (r.stage_bytes >> 1);
  c.tid = r.tid;
  c.nt = r.nt;
  return c;
}

// One run function: `BODY` runs the tile of one stage; the run goes on while the next item has
// the same run index.
// The state is copied into registers first: read through the reference, every field would be
// reloaded from the caller's local memory after each inline-asm memory clobber (a global-latency
// load per field per item, most of them L1 misses beside a large shared-memory carve-out).
#define GPUOS_RUN_LOOP(IDX, BODY)                                  \
  RunState rl = r;                                                 \
  uint32_t s = rl.s, parity = rl.parity;                           \
  uint64_t iter = rl.iter;                                         \
  do {                                                             \
    const TileCtx c = run_ctx(rl, s);                              \
    BODY;                                                          \
  } while (run_advance(rl, s, parity, iter, (IDX)));               \
  r.s = s;                                                         \
  r.parity = parity;                                               \
  r.iter = iter;                                                   \
  r.status = rl.status;

template <int OP>
__device__ __noinline__ void contig_run(RunState& r) { GPUOS_RUN_LOOP(OP, ew_contig<OP>(c)) }
template <int OP>
__device__ __noinline__ void t2d_run(RunState& r) { GPUOS_RUN_LOOP(kRunT2d + OP, ew_2dt<OP>(c)) }
template <int OP>
__device__ __noinline__ void e2d_run(RunState& r) { GPUOS_RUN_LOOP(kRun2d + OP, ew_2d<OP>(c)) }
__device__ __noinline__ void generic_run(RunState& r) { GPUOS_RUN_LOOP(kRunGeneric, ew_generic(c)) }
__device__ __noinline__ void t2d_shared_run(RunState& r) { GPUOS_RUN_LOOP(kRunT2dShared, ew_2dt<kDynOp>(c)) }
__device__ __noinline__ void reduce_run(RunState& r) {
  GPUOS_RUN_LOOP(GPUOS_EW_NUM_OPS, if (c.m->item.kind == IK_TOPK) topk_tile(c); else red_generic_tile(c))
}
#undef GPUOS_RUN_LOOP

typedef void (*RunFn)(RunState&);
#define GPUOS_RUN10(F, b) F<b + 0>, F<b + 1>, F<b + 2>, F<b + 3>, F<b + 4>, F<b + 5>, F<b + 6>, F<b + 7>, F<b + 8>, F<b + 9>
#define GPUOS_RUN30(F) GPUOS_RUN10(F, 0), GPUOS_RUN10(F, 10), GPUOS_RUN10(F, 20)
static_assert(GPUOS_EW_NUM_OPS == 30, "one run function per op in each group of g_run_fns");
__device__ RunFn g_run_fns[3 * GPUOS_EW_NUM_OPS + 3] = {GPUOS_RUN30(contig_run), reduce_run, GPUOS_RUN30(t2d_run),
                                                        GPUOS_RUN30(e2d_run), generic_run, t2d_shared_run};
#undef GPUOS_RUN30
#undef GPUOS_RUN10

__device__ __forceinline__ void compute_loop(const WorkerParams& P, const WorkerShared& W, uint32_t ctid, uint32_t nct) {
  SmemHeader& H = *W.H;
  const uint32_t S = P.stages;
  // plain registers: counters reached through a pointer would live in local memory and cost every
  // compute thread a local load and store per item
  unsigned long long wait_c = 0, tile_c = 0, fill_c = 0;
  uint32_t s = 0, parity = 0;  // stage and phase parity of use `iter` (stages are used in order)
  uint64_t iter = 0;
  bool ready = false;  // a run already waited for stage s to fill
  for (;;) {
    const unsigned long long c0 = clock64();
    if (!ready) {
      uint64_t waited = 0;
      if (!wait_phase(ptx::smem_addr(&H.full[s]), parity, &H.prod_alive, H.full_wait_ns, &waited)) {
        report_error(P, DE_WAIT_FULL, iter, waited, H.full_wait_ns);
        compute_diag(P, ctid, wait_c, tile_c, fill_c);
        return;
      }
    }
    ready = false;
    const StageMeta& m = H.meta[s];
    const uint8_t kind = m.item.kind;
    const unsigned long long c1 = clock64();
    wait_c += c1 - c0;
    if (ctid == 0 && (kind == IK_EW_CONTIG || kind == IK_ROW_REDUCE) && m.staged) fill_c += c1 - m.t_issue;
    if (kind == IK_EXIT) {
      compute_diag(P, ctid, wait_c, tile_c, fill_c);
      return;
    }
    if (kind == IK_TASK) {
      ptx::named_bar_sync(kBarTask, blockDim.x);
      OpFn fn = reinterpret_cast<OpFn>(m.item.x);
      fn(m.ext.task);
      ptx::named_bar_sync(kBarTask, blockDim.x);
    } else {
      const unsigned char* sa = stage_buf(W, s);
      const unsigned char* sb = sa + (W.stage_bytes >> 1);
      const bool first = iter == 0;
      if (first && ctid == 0) tl_mark(P, TL_TILE0);
      // inlined paths first (no register saves around a call)
      if (kind == IK_EW_CONTIG && f32_staged_tile(m, sa, sb, ctid, nct)) {
      } else if (kind == IK_ROW_REDUCE) {
        TileCtx ctx;
        ctx.m = &m;
        ctx.sa = sa;
        ctx.sb = sb;
        ctx.tid = ctid;
        ctx.nt = nct;
        row_reduce_body(ctx);
      } else {
        // a run of table tiles: it ends every tile it runs and leaves stage s filled
        const int idx = run_index(m);
        RunState r;
        r.P = &P;
        r.H = &H;
        r.bufs = W.bufs;
        r.stage_bytes = W.stage_bytes;
        r.S = S;
        r.s = s;
        r.parity = parity;
        r.iter = iter;
        r.tid = ctid;
        r.nt = nct;
        r.status = kRunNext;
        g_run_fns[idx < 0 ? GPUOS_EW_NUM_OPS : idx](r);
        if (first && ctid == 0) tl_mark(P, TL_TILE1);
        s = r.s;
        parity = r.parity;
        iter = r.iter;
        tile_c += clock64() - c1;
        if (r.status == kRunError) {
          compute_diag(P, ctid, wait_c, tile_c, fill_c);
          return;
        }
        ready = true;
        continue;
      }
      if (first && ctid == 0) tl_mark(P, TL_TILE1);
    }
    // this warp is done with the stage; no CTA-wide barrier between tiles
    __syncwarp();
    if ((ctid & 31) == 0) ptx::mbar_arrive(ptx::smem_addr(&H.done[s]));
    tile_c += clock64() - c1;
    ++iter;
    s = s + 1 == S ? 0 : s + 1;
    if (s == 0) parity ^= 1u;
  }
}

// ---- completer warp ------------------------------------------------------------------------
// Follows the stages in order: once every compute warp has signalled `done`, it hands the
// stage back to the dequeue warp and batches the completion accounting of several items
// behind one fence.  Before it would block on a stage the dequeue warp has not armed yet (no
// more work staged) it publishes what it has, so a lone item is accounted immediately; while
// armed stages are still loading or computing it keeps batching (an account is a gpu-scope fence
// and two contended atomics, and the next stage's release would wait behind it).
__device__ __forceinline__ void completer_loop(const WorkerParams& P, const WorkerShared& W, uint32_t lane) {
  SmemHeader& H = *W.H;
  const uint32_t S = P.stages;
  DoneRun runs[kMaxRuns];
  int nruns = 0;
  bool first_account = true;
  uint32_t pending = 0;
  const uint32_t acc_every = P.account_every ? P.account_every : kAccountEvery;
  unsigned long long t_wait = 0, t_acc = 0, n_items = 0;
  uint32_t s = 0, parity = 0;  // stage and phase parity of use `iter`
  for (uint64_t iter = 0;; ++iter, s = s + 1 == S ? 0 : s + 1, parity ^= s == 0 ? 1u : 0u) {
    int kind = 0;
    uint32_t batch = 0, batch_items = 0, batch_seq = 0;
    if (lane == 0) {
      unsigned long long c0 = clock64();
      const uint32_t full = ptx::smem_addr(&H.full[s]);
      const uint32_t armed = *reinterpret_cast<volatile unsigned int*>(&H.armed);
      if (nruns && (int32_t)(armed - (uint32_t)iter) <= 0 && !ptx::mbar_test_wait(full, parity)) {
        unsigned long long a0 = clock64();
        account(P, runs, nruns, &first_account);
        t_acc += clock64() - a0;
        nruns = 0;
        pending = 0;
      }
      uint64_t waited = 0;
      if (!wait_phase(full, parity, &H.prod_alive, H.full_wait_ns, &waited)) {
        report_error(P, DE_WAIT_FULL, iter, waited, H.full_wait_ns);
        kind = IK_EXIT;
      } else {
        const WorkItem& it = H.meta[s].item;
        kind = it.kind;
        batch = it.batch;
        batch_items = it.batch_items;
        batch_seq = it.batch_seq;
      }
      t_wait += clock64() - c0;
    }
    kind = __shfl_sync(0xffffffffu, kind, 0);
    if (kind == IK_EXIT) break;
    if (kind == IK_TASK) {
      ptx::named_bar_sync(kBarTask, blockDim.x);
      OpFn fn = reinterpret_cast<OpFn>(H.meta[s].item.x);
      fn(H.meta[s].ext.task);
      ptx::named_bar_sync(kBarTask, blockDim.x);
    }
    if (lane == 0) {
      unsigned long long c0 = clock64();
      const uint32_t done = ptx::smem_addr(&H.done[s]);
      const uint32_t armed = *reinterpret_cast<volatile unsigned int*>(&H.armed);
      if (nruns && (int32_t)(armed - (uint32_t)(iter + 1)) <= 0 && !ptx::mbar_test_wait(done, parity)) {
        account(P, runs, nruns, &first_account);
        nruns = 0;
        pending = 0;
      }
      uint64_t waited = 0;
      bool ok = wait_phase(done, parity, &H.prod_alive, H.full_wait_ns, &waited);
      unsigned long long c1 = clock64();
      t_wait += c1 - c0;
      if (!ok) {
        report_error(P, DE_WAIT_DONE, iter, waited, H.full_wait_ns);
      } else {
        ptx::mbar_arrive(ptx::smem_addr(&H.empty[s]));  // stage back to the dequeue warp
        if (nruns && runs[nruns - 1].batch == batch && runs[nruns - 1].batch_seq == batch_seq) {
          runs[nruns - 1].n += 1;
        } else {
          runs[nruns++] = DoneRun{batch, batch_items, batch_seq, 1u};
        }
        ++pending;
        ++n_items;
        if (pending >= acc_every || nruns == kMaxRuns) {
          account(P, runs, nruns, &first_account);
          nruns = 0;
          pending = 0;
        }
        t_acc += clock64() - c1;
      }
    }
    __syncwarp();
  }
  if (lane == 0) {
    if (nruns) account(P, runs, nruns, &first_account);
    if (blockIdx.x < kDiagCtas) {
      P.dc->diag[blockIdx.x][DG_C_BAR] = t_wait;
      P.dc->diag[blockIdx.x][DG_C_COMPLETE] = t_acc;
    }
  }
}

// ---- dequeue warp -------------------------------------------------------------------------
constexpr uint32_t kChunk = 8;  // tickets claimed per atomic when work is plentiful (dcache size)
constexpr int kDgTma = 6;       // ProdCold::dg index of the bulk-copy issue cycles (slot DG_P_TMA)

// Per-item state of the dequeue warp (registers; identical in every lane after each step).
struct ProdState {
  uint64_t iter;        // items staged so far
  uint64_t ticket;      // lowest unprocessed ticket held
  uint64_t chunk_end;   // tickets [ticket, chunk_end) are claimed by this CTA
  uint64_t desc_end;    // descriptors of tickets < desc_end are in dcache[cur]
  uint64_t n_ticket;    // chunk claimed ahead: tickets [n_ticket, n_end) (empty if equal)
  uint64_t n_end;
  uint64_t tail_cache;
  uint64_t items_done_cache;
  uint32_t n_fetched;   // the ahead chunk's descriptors are being copied into dcache[cur ^ 1]
  uint32_t cur;         // dcache buffer of the current chunk
  uint32_t last_seq;    // flush of the last staged item (start stamp once per flush)
  uint32_t stage;       // stage of use `iter`
  uint32_t phase;       // phase parity of use `iter` ((iter / S) & 1)
};

// Advance the stage cursor of the dequeue warp by n uses (n <= S).
__device__ __forceinline__ void advance(ProdState& st, uint32_t n, uint32_t S) {
  st.iter += n;
  st.stage += n;
  if (st.stage >= S) {
    st.stage -= S;
    st.phase ^= 1u;
  }
}

__device__ __forceinline__ void publish_diag(const WorkerParams& P, const ProdCold& C) {
  ptx::st_relaxed_sys(&P.rep->heartbeat, C.polls);
  ptx::st_relaxed_sys(&P.rep->head_mirror, *reinterpret_cast<volatile unsigned long long*>(&P.dc->head));
  ptx::st_relaxed_sys(&P.rep->items_done, *reinterpret_cast<volatile unsigned long long*>(&P.dc->items_done));
  ptx::st_relaxed_sys(&P.rep->park_rounds, C.rounds);
  ptx::st_relaxed_sys(&P.rep->park_timeouts, C.timeouts);
  ptx::st_relaxed_sys(&P.rep->park_work, C.work_resumes);
  ptx::st_relaxed_sys(&P.rep->parked_seen, C.parked_seen);
  ptx::st_relaxed_sys(&P.rep->host_read_ns_max, C.read_max);
  ptx::st_relaxed_sys(&P.rep->host_read_ns_avg, C.read_n ? C.read_sum / C.read_n : 0);
}

// Wait (lane 0) until stage `s` is free for use `iter` (whose phase parity is `phase`): the
// empty barrier of the stage completes phase (iter / S - 1) once use iter - S is released.
__device__ __forceinline__ bool wait_empty(const WorkerParams& P, SmemHeader& H, uint64_t iter, uint32_t s,
                                           uint32_t phase, uint32_t S) {
  if (iter < S) return true;
  const uint32_t parity = phase ^ 1u;
  const uint32_t bar = ptx::smem_addr(&H.empty[s]);
  const uint64_t t0 = ptx::now_ns();
  uint32_t spins = 0;
  while (!ptx::mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0) {
      const uint64_t t = ptx::now_ns();
      *reinterpret_cast<volatile unsigned long long*>(&H.prod_alive) = t;
      if (ptx::elapsed(t, t0) > H.wait_limit_ns) {
        report_error(P, DE_WAIT_EMPTY, iter, ptx::elapsed(t, t0), H.wait_limit_ns);
        return false;
      }
    }
  }
  return true;
}

// Wait (lane 0) until all `iter` staged items have been released by the compute warps.
__device__ __forceinline__ bool drain_own(const WorkerParams& P, SmemHeader& H, uint64_t iter, uint32_t S) {
  const uint64_t lo = iter > S ? iter - S : 0;
  for (uint64_t u = lo; u < iter; ++u) {
    // use u was released when the empty barrier of its stage completed phase (u / S)
    const uint32_t s = (uint32_t)(u % S);
    const uint32_t parity = (uint32_t)((u / S) & 1);
    const uint32_t bar = ptx::smem_addr(&H.empty[s]);
    const uint64_t t0 = ptx::now_ns();
    uint32_t spins = 0;
    while (!ptx::mbar_try_wait(bar, parity)) {
      if ((++spins & 255u) == 0 && ptx::elapsed(ptx::now_ns(), t0) > H.wait_limit_ns) {
        report_error(P, DE_WAIT_EMPTY, u);
        return false;
      }
    }
  }
  return true;
}

enum ParkVerdict { PV_RESUME = 1, PV_EXIT = 2 };
constexpr uint64_t kGatherNs = 200ull * 1000;  // leader gathers parked CTAs this long, then retries

// CTAs whose parked flag shows `round` (the leader's scan: independent loads, 16 in flight).
__device__ __forceinline__ uint32_t count_parked(DevCtl* dc, uint64_t round) {
  const uint32_t n = gridDim.x;
  uint32_t cnt = 0;
  for (uint32_t c0 = 0; c0 < n; c0 += 16) {
    unsigned long long v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = c0 + k < n ? ptx::ld_relaxed_gpu(&dc->parked[c0 + k]) : ~0ull;
#pragma unroll
    for (int k = 0; k < 16; ++k) cnt += v[k] == round ? 1u : 0u;
  }
  return cnt;
}

// Park protocol (lane 0 of a dequeue warp that is idle and holds an unpublished ticket).
// Returns PV_RESUME or PV_EXIT.
__device__ __forceinline__ int park(const WorkerParams& P, SmemHeader& H, const ProdState& st, uint64_t round,
                                    uint32_t S) {
  DevCtl* dc = P.dc;
  ProdCold& C = H.cold;
  C.seen_round = round;
  const bool leader = blockIdx.x == 0;
  if (!leader) {
    const unsigned long long v = ptx::ld_acquire_gpu(&dc->verdict);
    if ((v >> 2) == round) return (int)(v & 3);
    if ((v >> 2) > round) return PV_RESUME;
  }
  if (!drain_own(P, H, st.iter, S)) return PV_EXIT;
  atomicMin(&dc->park_min, (unsigned long long)st.ticket);
  ptx::st_release_gpu(&dc->parked[blockIdx.x], round);
  const uint64_t t0 = ptx::now_ns();
  if (leader) {
    uint32_t spins = 0;
    bool gathered = false;
    while (true) {
      if (count_parked(dc, round) >= gridDim.x) {
        ptx::fence_acq_rel_gpu();  // every parked CTA's park_min update is visible from here on
        gathered = true;
        break;
      }
      if (*reinterpret_cast<volatile unsigned int*>(&dc->abort)) break;
      const uint64_t t = ptx::ld_acquire_sys(&P.hc->tail);
      if (t > *reinterpret_cast<volatile unsigned long long*>(&dc->park_min)) {  // work for a parked CTA
        ++C.work_resumes;
        break;
      }
      if ((++spins & 15u) == 0) {
        const uint64_t now = ptx::now_ns();
        *reinterpret_cast<volatile unsigned long long*>(&H.prod_alive) = now;
        if (ptx::elapsed(now, t0) > kGatherNs) {  // someone is still busy: retry later
          ++C.timeouts;
          C.parked_seen = count_parked(dc, round);
          break;
        }
      }
      ptx::nanosleep(128);
    }
    if (C.rounds == 1) tl_mark(P, TL_GATHER);
    const bool aborted = *reinterpret_cast<volatile unsigned int*>(&dc->abort) != 0;
    if (!gathered && !aborted) {
      C.mirrored = ptx::ld_acquire_sys(&P.hc->tail);
      ptx::st_release_gpu(&dc->tail_mirror, C.mirrored);
      ptx::st_release_gpu(&dc->verdict, (round << 2) | PV_RESUME);
      return PV_RESUME;
    }
    // Publish EXITING, then re-read the host tail: the host stores tail, fences, then
    // reads the state, so at least one side sees the other's write.
    ptx::st_relaxed_sys(&P.rep->state, (P.epoch << 8) | WS_EXITING);
    ptx::fence_sc_sys();
    const uint64_t T = ptx::ld_acquire_sys(&P.hc->tail);
    const uint64_t pm = *reinterpret_cast<volatile unsigned long long*>(&dc->park_min);
    if (!aborted && T > pm) {
      ++C.work_resumes;
      ptx::st_relaxed_sys(&P.rep->state, (P.epoch << 8) | WS_RUNNING);
      ptx::st_release_gpu(&dc->tail_mirror, T);
      C.mirrored = T;
      ptx::st_release_gpu(&dc->verdict, (round << 2) | PV_RESUME);
      return PV_RESUME;
    }
    dc->exit_tail = pm;
    publish_diag(P, C);
    tl_mark(P, TL_VERDICT);
    ptx::st_release_gpu(&dc->verdict, (round << 2) | PV_EXIT);
    return PV_EXIT;
  }
  uint32_t spins = 0;
  while (true) {
    const unsigned long long v = ptx::ld_acquire_gpu(&dc->verdict);
    if ((v >> 2) == round) return (int)(v & 3);
    if ((v >> 2) > round) return PV_RESUME;
    if (*reinterpret_cast<volatile unsigned int*>(&dc->abort)) return PV_EXIT;
    if ((++spins & 63u) == 0) {
      const uint64_t now = ptx::now_ns();
      *reinterpret_cast<volatile unsigned long long*>(&H.prod_alive) = now;
      if (ptx::elapsed(now, t0) > H.wait_limit_ns) {
        report_error(P, DE_WAIT_PARK, st.ticket, ptx::elapsed(now, t0), H.wait_limit_ns);
        return PV_EXIT;
      }
    }
    ptx::nanosleep(256);
  }
}

// Copy `bytes` (multiple of 16) from mapped/global memory into shared memory with the warp.
__device__ __forceinline__ void warp_copy16(void* dst, const void* src, uint32_t bytes, uint32_t lane) {
  for (uint32_t off = lane * 16; off < bytes; off += 32 * 16) {
    const uint4 v = ptx::ld_cg_v4(reinterpret_cast<const unsigned char*>(src) + off);
    *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(dst) + off) = v;
  }
}

// Copy `bytes` (multiple of 16) within shared memory with the warp.
__device__ __forceinline__ void warp_copy_smem16(void* dst, const void* src, uint32_t bytes, uint32_t lane) {
  for (uint32_t off = lane * 16; off < bytes; off += 32 * 16)
    *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(dst) + off) =
        *reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(src) + off);
}

// Arm stage s as the exit sentinel (lane 0).
__device__ __forceinline__ void arm_exit(SmemHeader& H, uint32_t s) {
  H.meta[s].item.kind = IK_EXIT;
  ptx::mbar_arrive(ptx::smem_addr(&H.full[s]));
}

// Items the group path stages without help: contiguous element-wise tiles and row groups.
__device__ __forceinline__ bool group_kind(const WorkItem& it) {
  return it.batch < kNumBatchSlots &&
         ((it.kind == IK_EW_CONTIG && it.op < GPUOS_EW_NUM_OPS) || it.kind == IK_ROW_REDUCE);
}

// Issue the operand copies of a contiguous element-wise tile or a row group into stage s
// and arrive on its full barrier (one thread).  m.item is already written.
__device__ __forceinline__ void stage_copies(const WorkerShared& W, StageMeta& m, uint32_t s, const WorkItem& it) {
  const uint32_t full = ptx::smem_addr(&W.H->full[s]);
  m.t_issue = clock64();
  unsigned char* buf = stage_buf(W, s);
  uint32_t staged = 0;
  if (it.kind == IK_EW_CONTIG) {
    uint32_t tx = 0;
    uint64_t a0 = 0, a1 = 0, b0 = 0, b1 = 0;
    const uint32_t half = W.stage_bytes >> 1;
    if (!(it.flags & IF_A_BCAST)) {
      const uint64_t bytes = (uint64_t)it.count * dtype_size(it.dt_a);
      a0 = it.a & ~15ull;
      a1 = (it.a + bytes + 15) & ~15ull;
      if (a1 - a0 <= half) {
        m.a_off = (uint32_t)(it.a - a0);
        staged |= 1;
        tx += (uint32_t)(a1 - a0);
      }
    }
    if ((it.flags & IF_B_PRESENT) && !(it.flags & (IF_B_SCALAR | IF_B_BCAST))) {
      const uint64_t bytes = (uint64_t)it.count * dtype_size(it.dt_b);
      b0 = it.b & ~15ull;
      b1 = (it.b + bytes + 15) & ~15ull;
      if (b1 - b0 <= half) {
        m.b_off = (uint32_t)(it.b - b0);
        staged |= 2;
        tx += (uint32_t)(b1 - b0);
      }
    }
    m.staged = staged;
    if (tx) {
      ptx::mbar_arrive_expect_tx(full, tx);
      if (W.load_policy) {
        if (staged & 1)
          ptx::bulk_g2s_hint(ptx::smem_addr(buf), reinterpret_cast<const void*>(a0), (uint32_t)(a1 - a0), full,
                             W.load_policy);
        if (staged & 2)
          ptx::bulk_g2s_hint(ptx::smem_addr(buf + half), reinterpret_cast<const void*>(b0), (uint32_t)(b1 - b0), full,
                             W.load_policy);
      } else {
        if (staged & 1) ptx::bulk_g2s(ptx::smem_addr(buf), reinterpret_cast<const void*>(a0), (uint32_t)(a1 - a0), full);
        if (staged & 2)
          ptx::bulk_g2s(ptx::smem_addr(buf + half), reinterpret_cast<const void*>(b0), (uint32_t)(b1 - b0), full);
      }
    } else {
      ptx::mbar_arrive(full);
    }
  } else if (it.kind == IK_ROW_REDUCE && !(it.flags & IF_UNSTAGED)) {
    const int es = dtype_size(it.dt_a);
    const int64_t rows = it.count, C = it.aux, rs = (int64_t)it.x, is = (int64_t)it.b;
    const uint64_t span = (uint64_t)(((rows - 1) * rs + (C - 1) * is + 1) * es);
    const uint64_t a0 = it.a & ~15ull;
    const uint64_t a1 = (it.a + span + 15) & ~15ull;
    if (a1 - a0 <= W.stage_bytes) {
      m.a_off = (uint32_t)(it.a - a0);
      m.staged = 1;
      ptx::mbar_arrive_expect_tx(full, (uint32_t)(a1 - a0));
      ptx::bulk_g2s(ptx::smem_addr(buf), reinterpret_cast<const void*>(a0), (uint32_t)(a1 - a0), full);
    } else {
      m.staged = 0;
      ptx::mbar_arrive(full);
    }
  } else if (it.kind == IK_EW_2DT) {
    // every row of the block x its columns: one contiguous span of a (layout already copied)
    const Layout& L = m.ext.layout;
    const uint64_t nr = it.count >> 16, nc = it.count & 0xffffu, c0 = it.x >> 32;
    const uint64_t es = (uint64_t)dtype_size(it.dt_a);
    const uint64_t start = it.a + c0 * (uint64_t)L.sa[1] * es;
    const uint64_t span = ((nc - 1) * (uint64_t)L.sa[1] + nr) * es;
    const uint64_t a0 = start & ~15ull;
    const uint64_t a1 = (start + span + 15) & ~15ull;
    if (L.sa[0] == 1 && L.sa[1] > 0 && nc > 0 && a1 - a0 <= (W.stage_bytes >> 1)) {
      m.a_off = (uint32_t)(start - a0);
      m.staged = 1;
      ptx::mbar_arrive_expect_tx(full, (uint32_t)(a1 - a0));
      if (W.load_policy)
        ptx::bulk_g2s_hint(ptx::smem_addr(buf), reinterpret_cast<const void*>(a0), (uint32_t)(a1 - a0), full,
                           W.load_policy);
      else
        ptx::bulk_g2s(ptx::smem_addr(buf), reinterpret_cast<const void*>(a0), (uint32_t)(a1 - a0), full);
    } else {
      m.staged = 0;
      ptx::mbar_arrive(full);
    }
  } else if (it.kind == IK_TOPK) {
    const uint64_t span = (uint64_t)it.count * it.aux * dtype_size(it.dt_a);
    const uint64_t a0 = it.a & ~15ull;
    const uint64_t a1 = (it.a + span + 15) & ~15ull;
    if (a1 - a0 <= W.stage_bytes) {
      m.a_off = (uint32_t)(it.a - a0);
      m.staged = 1;
      ptx::mbar_arrive_expect_tx(full, (uint32_t)(a1 - a0));
      ptx::bulk_g2s(ptx::smem_addr(buf), reinterpret_cast<const void*>(a0), (uint32_t)(a1 - a0), full);
    } else {
      m.staged = 0;
      ptx::mbar_arrive(full);
    }
  } else {
    m.staged = 0;
    ptx::mbar_arrive(full);
  }
}

// Stage the item of st.ticket alone (whole dequeue warp; stage `st.iter % S` is free): every
// kind, dependency barriers, malformed items.  On an error the stage is armed as the exit
// sentinel and false is returned.
__device__ __forceinline__ bool stage_item(const WorkerParams& P, const WorkerShared& W, ProdState& st, uint32_t lane) {
  SmemHeader& H = *W.H;
  const uint32_t S = P.stages;
  const uint32_t s = st.stage;
  StageMeta& m = H.meta[s];
  if (lane == 0 && st.iter == 0) tl_mark(P, TL_STAGE);
  if (lane < 4) {
    const uint4* src = reinterpret_cast<const uint4*>(&H.dcache[st.cur][st.ticket & 7]);
    reinterpret_cast<uint4*>(&m.item)[lane] = src[lane];
  }
  __syncwarp();
  const WorkItem it = m.item;
  int ok = 1;
  if (lane == 0) {
    if (it.kind == IK_NONE || it.kind > IK_EW_2DT || it.batch >= kNumBatchSlots ||
        (it.kind != IK_TASK && it.kind != IK_ROW_REDUCE && it.kind != IK_RED_GENERIC && it.op >= GPUOS_EW_NUM_OPS)) {
      report_error(P, DE_BAD_ITEM, st.ticket);
      ok = 0;
    }
    // dependency barrier: every item before the segment start must be complete
    if (ok && it.wait_items > st.items_done_cache) {
      const uint64_t t0 = ptx::now_ns();
      uint32_t spins = 0;
      while (true) {
        st.items_done_cache = ptx::ld_acquire_gpu(&P.dc->items_done);
        if (st.items_done_cache >= it.wait_items) break;
        if (*reinterpret_cast<volatile unsigned int*>(&P.dc->abort)) { ok = 0; break; }
        if ((++spins & 63u) == 0) {
          const uint64_t now = ptx::now_ns();
          *reinterpret_cast<volatile unsigned long long*>(&H.prod_alive) = now;
          if (ptx::elapsed(now, t0) > H.wait_limit_ns) {
            report_error(P, DE_WAIT_BARRIER, st.ticket, ptx::elapsed(now, t0), H.wait_limit_ns);
            ok = 0;
            break;
          }
        }
        ptx::nanosleep(64);
      }
    }
    // start stamp of the flush: the first item each CTA stages from it is enough
    if (ok && it.batch_seq != st.last_seq) {
      atomicMin(&P.dc->batch_t0[it.batch], (unsigned long long)ptx::now_ns());
      st.last_seq = it.batch_seq;
    }
    if (!ok) arm_exit(H, s);
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  st.items_done_cache = __shfl_sync(0xffffffffu, st.items_done_cache, 0);
  st.last_seq = __shfl_sync(0xffffffffu, st.last_seq, 0);
  if (!ok) return false;

  if (it.kind == IK_EW_GENERIC || it.kind == IK_EW_2D || it.kind == IK_EW_2DT || it.kind == IK_RED_GENERIC) {
    if (H.lay_valid && H.lay_key == it.aux) {
      warp_copy_smem16(&m.ext.layout, &H.lay_cache, sizeof(Layout), lane);
    } else {
      warp_copy16(&m.ext.layout, P.layouts + (it.aux & P.layout_mask), sizeof(Layout), lane);
      __syncwarp();
      warp_copy_smem16(&H.lay_cache, &m.ext.layout, sizeof(Layout), lane);
      __syncwarp();
      if (lane == 0) {
        H.lay_key = it.aux;
        H.lay_valid = 1;
      }
    }
  } else if (it.kind == IK_TASK) {
    warp_copy16(&m.ext.task, P.tasks + (it.aux & P.task_mask), sizeof(Task), lane);
  }
  __syncwarp();
  if (lane == 0) {
    if (it.kind == IK_TASK) {
      m.staged = 0;
      const OpFn fn = resolve_op(P, m.ext.task.op);
      if (fn == nullptr) {
        report_error(P, DE_NULL_OP, st.ticket);
        ok = 0;
        arm_exit(H, s);
      } else {
        m.item.x = reinterpret_cast<uint64_t>(fn);
        ptx::mbar_arrive(ptx::smem_addr(&H.full[s]));
      }
    } else {
      stage_copies(W, m, s, it);
    }
    if (st.iter == 0) tl_mark(P, TL_TMA);
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) return false;
  if (it.kind == IK_TASK) {
    // run the reference-ABI operator with the whole CTA
    ptx::named_bar_sync(kBarTask, blockDim.x);
    OpFn fn = reinterpret_cast<OpFn>(m.item.x);
    fn(m.ext.task);
    ptx::named_bar_sync(kBarTask, blockDim.x);
  }
  advance(st, 1, S);
  st.ticket += 1;
  if (lane == 0) *reinterpret_cast<volatile unsigned int*>(&H.armed) = (uint32_t)st.iter;
  return true;
}

// Stage up to S items of the current chunk at once, one lane per item: the items whose
// descriptors are here, that the group path handles, need no dependency wait, and whose
// stages are already free (stage st.iter is).  Returns the number staged (0: the item of
// st.ticket needs stage_item).
__device__ __forceinline__ uint32_t stage_group(const WorkerParams& P, const WorkerShared& W, ProdState& st,
                                                uint32_t lane) {
  SmemHeader& H = *W.H;
  const uint32_t S = P.stages;
  const uint64_t have = st.desc_end - st.ticket;
  const uint32_t navail = (uint32_t)(have < S ? have : S);
  WorkItem it;
  bool ok = false;
  if (lane < navail) {
    it = H.dcache[st.cur][(st.ticket + lane) & 7];
    const uint64_t u = st.iter + lane;
    uint32_t su = st.stage + lane, ph = st.phase;
    if (su >= S) {
      su -= S;
      ph ^= 1u;
    }
    const bool free = lane == 0 || u < S || ptx::mbar_test_wait(ptx::smem_addr(&H.empty[su]), ph ^ 1u);
    // staged transpose blocks join the group once their layout record is cached here
    const bool t2d = it.kind == IK_EW_2DT && it.batch < kNumBatchSlots && it.op < GPUOS_EW_NUM_OPS &&
                     H.lay_valid && H.lay_key == it.aux;
    ok = free && (group_kind(it) || t2d) && it.wait_items <= st.items_done_cache;
  } else {
    it.batch_seq = 0;
  }
  const uint32_t mask = __ballot_sync(0xffffffffu, ok);
  const uint32_t g = (uint32_t)__ffs(~mask) - 1;  // leading lanes that can stage
  if (g == 0) return 0;
  const uint32_t prev_seq = __shfl_up_sync(0xffffffffu, it.batch_seq, 1);
  if (lane < g) {
    const uint32_t s = st.stage + lane < S ? st.stage + lane : st.stage + lane - S;
    StageMeta& m = H.meta[s];
    m.item = it;
    // start stamp of the flush: the first item each CTA stages from it is enough
    if (it.batch_seq != (lane == 0 ? st.last_seq : prev_seq))
      atomicMin(&P.dc->batch_t0[it.batch], (unsigned long long)ptx::now_ns());
    if (it.kind == IK_EW_2DT) {
      // the fields of the layout record a staged transpose block reads (not the whole record)
      Layout& L = m.ext.layout;
      const Layout& Lc = H.lay_cache;
      L.sa[0] = Lc.sa[0];
      L.sa[1] = Lc.sa[1];
      L.sb[0] = Lc.sb[0];
      L.sb[1] = Lc.sb[1];
      L.so[0] = Lc.so[0];
      L.so[1] = Lc.so[1];
      L.params[0] = Lc.params[0];
      L.params[1] = Lc.params[1];
    }
    stage_copies(W, m, s, it);
  }
  st.last_seq = __shfl_sync(0xffffffffu, it.batch_seq, g - 1);
  if (lane == 0 && st.iter == 0) {
    tl_mark(P, TL_STAGE);
    tl_mark(P, TL_TMA);
  }
  __syncwarp();
  advance(st, g, S);
  st.ticket += g;
  if (lane == 0) *reinterpret_cast<volatile unsigned int*>(&H.armed) = (uint32_t)st.iter;
  return g;
}

// Tickets per CTA share of `ahead` published tickets: ahead / (2 x grid), in 32 bits (a 64-bit
// division is a long software routine); at least kChunk whenever the quotient would be.
__device__ __forceinline__ uint64_t chunk_share(uint64_t ahead) {
  const uint32_t d = 2u * gridDim.x;
  return ahead >= (uint64_t)kChunk * d ? (uint64_t)kChunk : (uint64_t)((uint32_t)ahead / d);
}

__device__ __forceinline__ void producer_loop(const WorkerParams& P, const WorkerShared& W, uint32_t lane) {
  SmemHeader& H = *W.H;
  ProdCold& C = H.cold;
  DevCtl* dc = P.dc;
  const uint32_t S = P.stages;
  const bool leader = blockIdx.x == 0;
  ProdState st;
  st.iter = 0;
  st.ticket = 0;
  st.chunk_end = 0;
  st.desc_end = 0;
  st.n_ticket = st.n_end = 0;
  st.n_fetched = 0;
  st.cur = 0;
  st.last_seq = 0;
  st.stage = 0;
  st.phase = 0;
  st.tail_cache = ptx::ld_acquire_gpu(&dc->tail_mirror);
  st.items_done_cache = 0;
  if (lane == 0) {
    C.seen_round = 0;
    C.round = 0;
    C.beat_val = leader ? P.hc->host_beat : 0;
    C.beat_t = ptx::now_ns();
    C.polls = 0;
    C.quit_epoch = ptx::ld_acquire_gpu(&dc->p_quit_epoch);
    C.yield_every = ptx::ld_acquire_gpu(&dc->p_yield_every);
    C.safety_ns = ptx::ld_acquire_gpu(&dc->p_safety_idle_ns);
    C.spin_ns = ptx::ld_acquire_gpu(&dc->p_spin_ns);
    C.read_sum = C.read_n = C.read_max = 0;
    C.mirrored = st.tail_cache;
    H.lay_valid = 0;
    C.rounds = C.timeouts = C.work_resumes = C.parked_seen = 0;
    for (int k = 0; k < 7; ++k) C.dg[k] = 0;
  }
  __syncwarp();

  while (true) {
    int action = 0;  // 0: stage, 1: exit, 2: error after staging began
    uint32_t switched = 0, issue = 0;
    if (lane == 0) {
      unsigned long long c0 = clock64();
      const bool empty_ok = wait_empty(P, H, st.iter, st.stage, st.phase, S);
      unsigned long long c1 = clock64();
      C.dg[DG_P_WAIT_EMPTY] += c1 - c0;
      if (!empty_ok) {
        action = 1;
      } else if (st.ticket == st.chunk_end) {
        if (st.n_end > st.n_ticket) {
          // move on to the chunk claimed ahead
          st.ticket = st.n_ticket;
          st.chunk_end = st.n_end;
          st.desc_end = st.n_fetched ? st.n_end : st.n_ticket;
          switched = st.n_fetched;
          st.n_ticket = st.n_end = 0;
          st.n_fetched = 0;
        } else {
          // Claim a chunk: several tickets per atomic while plenty of published work lies
          // ahead, single tickets near the end of the published work (load balance).
          const uint64_t ahead = st.tail_cache > st.chunk_end ? st.tail_cache - st.chunk_end : 0;
          uint64_t k = chunk_share(ahead);
          k = k < 1 ? 1 : (k > kChunk ? kChunk : k);
          if (st.iter == 0 && st.chunk_end == 0) tl_mark(P, TL_CLAIM);
          st.ticket = atomicAdd(&dc->head, k);
          st.chunk_end = st.ticket + k;
          st.desc_end = st.ticket;
        }
        // Claim the next chunk now while at least two tickets per CTA of published work lie
        // beyond this one; its descriptors are copied while this chunk is staged.  A CTA
        // that goes idle never holds a chunk ahead (this chunk would have to be published).
        const uint64_t ahead = st.tail_cache > st.chunk_end ? st.tail_cache - st.chunk_end : 0;
        if (st.chunk_end <= st.tail_cache && ahead >= 2ull * gridDim.x) {
          uint64_t k = chunk_share(ahead);
          k = k > kChunk ? kChunk : k;
          st.n_ticket = atomicAdd(&dc->head, k);
          st.n_end = st.n_ticket + k;
          st.n_fetched = st.n_end <= st.tail_cache;
          issue = st.n_fetched;
        }
        c0 = clock64();
        C.dg[DG_P_CLAIM] += c0 - c1;
        c1 = c0;
      }
      while (action == 0 && st.ticket >= st.tail_cache) {
        // idle: poll for publication, watch for exit conditions.  The control words are
        // loaded first and the tail (acquire) last, so one poll costs one round trip.
        ++C.polls;
        const unsigned int ab = *reinterpret_cast<volatile unsigned int*>(&dc->abort);
        unsigned long long cl = ptx::ld_relaxed_gpu(&dc->closing);
        const bool ctl = leader && (C.polls & 7u) == 0;  // host control words: every few polls
        uint64_t q = 0, beat = 0;
        if (ctl) {
          q = ptx::ld_relaxed_sys(&P.hc->quit_epoch);
          beat = ptx::ld_relaxed_sys(&P.hc->host_beat);
        }
        uint64_t t;
        if (leader) {
          // only the leader reads host memory; everybody else polls its device mirror
          const uint64_t r0 = ptx::now_ns();
          t = ptx::ld_acquire_sys(&P.hc->tail);
          const uint64_t dr = ptx::elapsed(ptx::now_ns(), r0);
          C.read_sum += dr;
          ++C.read_n;
          if (dr > C.read_max) C.read_max = dr;
          if (t > C.mirrored) {
            ptx::st_release_gpu(&dc->tail_mirror, t);
            C.mirrored = t;
          }
        } else {
          t = ptx::ld_acquire_gpu(&dc->tail_mirror);
        }
        if (st.ticket < t) {
          st.tail_cache = t;
          break;
        }
        const uint64_t now = ptx::now_ns();
        *reinterpret_cast<volatile unsigned long long*>(&H.prod_alive) = now;
        if (ab) {
          action = 1;
          break;
        }
        if (leader) {
          if (ctl) {
            C.quit_epoch = q;
            if (beat != C.beat_val) {
              C.beat_val = beat;
              C.beat_t = now;
            }
            if ((C.polls & 63u) == 0) {
              C.yield_every = P.hc->yield_every;
              C.safety_ns = P.hc->safety_idle_ns;
              C.spin_ns = P.hc->spin_ns;
              publish_diag(P, C);
            }
          }
          bool want_exit = C.quit_epoch >= P.epoch;
          if (want_exit) {
            // the host withdraws an idle stop when it publishes work: confirm before exiting
            C.quit_epoch = P.hc->quit_epoch;
            want_exit = C.quit_epoch >= P.epoch;
          }
          if (C.yield_every && ptx::ld_acquire_gpu(&dc->items_done) - dc->yield_base >= C.yield_every) want_exit = true;
          if (ptx::elapsed(now, C.beat_t) > C.safety_ns) want_exit = true;
          if (want_exit) {
            C.round = (C.round > C.seen_round ? C.round : C.seen_round) + 1;
            if (C.rounds == 0) tl_mark(P, TL_ROUND);
            ++C.rounds;
            atomicExch(&dc->park_min, ~0ull);
            ptx::fence_acq_rel_gpu();
            ptx::st_release_gpu(&dc->closing, C.round);
            cl = C.round;  // the leader joins its own round at once
          }
        }
        if (cl > C.seen_round) {
          ptx::fence_acq_rel_gpu();  // with the relaxed load of `closing`: acquire of the round
          const int v = park(P, H, st, cl, S);
          if (v == PV_EXIT) {
            action = 1;
            break;
          }
          st.tail_cache = ptx::ld_acquire_gpu(&dc->tail_mirror);
          continue;
        }
        ptx::nanosleep(leader ? (uint32_t)C.spin_ns : 128);
      }
      C.dg[DG_P_IDLE] += clock64() - c1;
    }
    action = __shfl_sync(0xffffffffu, action, 0);
    if (action == 1) {
      if (lane == 0) {
        wait_empty(P, H, st.iter, st.stage, st.phase, S);
        arm_exit(H, st.stage);
      }
      break;
    }
    __syncwarp();  // orders lane 0's acquire of the tail before the other lanes' descriptor reads
    st.ticket = __shfl_sync(0xffffffffu, st.ticket, 0);
    st.chunk_end = __shfl_sync(0xffffffffu, st.chunk_end, 0);
    st.desc_end = __shfl_sync(0xffffffffu, st.desc_end, 0);
    st.tail_cache = __shfl_sync(0xffffffffu, st.tail_cache, 0);
    switched = __shfl_sync(0xffffffffu, switched, 0);
    issue = __shfl_sync(0xffffffffu, issue, 0);
    unsigned long long cd = clock64();
    if (switched) {
      // the chunk claimed ahead is current: wait for the copies of its descriptors
      ptx::cp_async_wait_all();
      __syncwarp();
      st.cur ^= 1u;
    }
    if (issue) {
      st.n_ticket = __shfl_sync(0xffffffffu, st.n_ticket, 0);
      st.n_end = __shfl_sync(0xffffffffu, st.n_end, 0);
      st.n_fetched = 1;
      if (lane < 4 * (uint32_t)(st.n_end - st.n_ticket)) {
        const uint64_t t = st.n_ticket + (lane >> 2);
        ptx::cp_async_cg16(ptx::smem_addr(&H.dcache[st.cur ^ 1u][t & 7]) + (lane & 3) * 16,
                           reinterpret_cast<const unsigned char*>(P.items + (t & P.item_mask)) + (lane & 3) * 16);
      }
      ptx::cp_async_commit();
    }
    if (st.ticket >= st.desc_end) {
      // one warp-wide read fetches the descriptors of every published ticket of the chunk
      const uint64_t hi = st.chunk_end < st.tail_cache ? st.chunk_end : st.tail_cache;
      const uint32_t cnt = (uint32_t)(hi - st.ticket);
      if (lane < 4 * cnt) {
        const uint64_t t = st.ticket + (lane >> 2);
        const unsigned char* src = reinterpret_cast<const unsigned char*>(P.items + (t & P.item_mask)) + (lane & 3) * 16;
        reinterpret_cast<uint4*>(&H.dcache[st.cur][t & 7])[lane & 3] = ptx::ld_cg_v4(src);
      }
      __syncwarp();
      st.desc_end = hi;
    }
    unsigned long long ce = clock64();
    if (lane == 0) C.dg[DG_P_DESC] += ce - cd;
    uint32_t g = stage_group(P, W, st, lane);
    if (g == 0) {
      if (!stage_item(P, W, st, lane)) break;
      g = 1;
    }
    if (lane == 0) {
      C.dg[DG_P_STAGE] += clock64() - ce;
      C.dg[DG_P_ITEMS] += g;
    }
  }
  // no descriptor copy may still be landing in shared memory when the warp leaves
  ptx::cp_async_wait_all();
  __syncwarp();
  if (lane == 0 && blockIdx.x < kDiagCtas) {
    unsigned long long* row = dc->diag[blockIdx.x];
    for (int k = 0; k < 6; ++k) row[k] = C.dg[k];

  }
}

// ---- the kernel ---------------------------------------------------------------------------
__device__ void batch_worker_body(const WorkerParams& P, unsigned char* smem_raw) {
  SmemHeader* H = reinterpret_cast<SmemHeader*>(smem_raw);
  WorkerShared W;
  W.H = H;
  W.bufs = smem_raw + ((sizeof(SmemHeader) + 127) & ~size_t(127));
  W.stage_bytes = P.stage_bytes;
  W.load_policy = P.load_hint ? ptx::l2_evict_first_policy() : 0ull;
  const uint32_t S = P.stages;
  DevCtl* dc = P.dc;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      ptx::mbar_init(ptx::smem_addr(&H->full[s]), 1);
      ptx::mbar_init(ptx::smem_addr(&H->empty[s]), 1);
      ptx::mbar_init(ptx::smem_addr(&H->done[s]), (blockDim.x - 64) / 32);
    }
    ptx::fence_mbar_init();
    H->prod_alive = ptx::now_ns();
    H->wait_limit_ns = P.wait_limit_ns;
    H->full_wait_ns = P.wait_limit_ns;
    H->exit_flag = 0;
    H->armed = 0;
  }
  __syncthreads();

  // Launch initialisation: CTA 0 resets the dequeue position to where the previous
  // launch stopped; the other CTAs wait for it (bounded).
  __shared__ int start_ok;
  if (threadIdx.x == 0) {
    start_ok = 1;
    if (blockIdx.x == 0) {
      dc->head = dc->exit_tail;
      dc->closing = 0;
      dc->verdict = 0;
      for (uint32_t c = 0; c < gridDim.x && c < (uint32_t)kDiagCtas; ++c) dc->parked[c] = 0;
      dc->park_min = ~0ull;
      dc->abort = 0;
      dc->exited = 0;
      dc->yield_base = dc->items_done;
      if (gridDim.x < kDiagCtas) {
        for (int k = 0; k < kDiagSlots; ++k) dc->diag[gridDim.x][k] = ~0ull;
        dc->diag[gridDim.x][TL_INIT] = ptx::now_ns();
      }
      dc->tail_mirror = ptx::ld_acquire_sys(&P.hc->tail);
      dc->p_wait_limit_ns = P.hc->wait_limit_ns;
      dc->p_safety_idle_ns = P.hc->safety_idle_ns;
      dc->p_yield_every = P.hc->yield_every;
      dc->p_quit_epoch = P.hc->quit_epoch;
      dc->p_spin_ns = P.hc->spin_ns;
      ptx::fence_acq_rel_gpu();
      ptx::st_release_gpu(&dc->launch_epoch, P.epoch);
      ptx::st_relaxed_sys(&P.rep->t_launch, ptx::now_ns());
      ptx::st_relaxed_sys(&P.rep->state, (P.epoch << 8) | WS_RUNNING);
      ptx::fence_acq_rel_sys();
      ptx::st_relaxed_sys(&P.rep->ready_epoch, P.epoch);
    } else {
      const uint64_t t0 = ptx::now_ns();
      while (ptx::ld_acquire_gpu(&dc->launch_epoch) != P.epoch) {
        if (ptx::elapsed(ptx::now_ns(), t0) > P.wait_limit_ns) {
          report_error(P, DE_WAIT_START, 0);
          start_ok = 0;
          break;
        }
        ptx::nanosleep(128);
      }
    }
    if (start_ok) {
      const uint64_t wl = ptx::ld_acquire_gpu(&dc->p_wait_limit_ns);
      H->wait_limit_ns = wl;
      H->full_wait_ns = wl + ptx::ld_acquire_gpu(&dc->p_safety_idle_ns);
    }
  }
  __syncthreads();
  const unsigned long long cta_c0 = clock64();
  if (start_ok) {
    const uint32_t warp = threadIdx.x >> 5;
    if (warp == 0) producer_loop(P, W, threadIdx.x & 31);
    else if (warp == 1) completer_loop(P, W, threadIdx.x & 31);
    else compute_loop(P, W, threadIdx.x - 64, blockDim.x - 64);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (blockIdx.x < kDiagCtas) dc->diag[blockIdx.x][DG_CYCLES] = clock64() - cta_c0;
    tl_mark(P, TL_EXIT_FIRST);
    ptx::fence_acq_rel_gpu();
    const unsigned int n = atomicAdd(&dc->exited, 1u) + 1;
    if (n == gridDim.x) {
      if (gridDim.x < kDiagCtas) dc->diag[gridDim.x][TL_EXIT_LAST] = ptx::now_ns();
      ptx::st_relaxed_sys(&P.rep->exit_tail, dc->exit_tail);
      ptx::st_relaxed_sys(&P.rep->t_exit, ptx::now_ns());
      ptx::st_relaxed_sys(&P.rep->items_done, dc->items_done);
      ptx::fence_sc_sys();
      ptx::st_relaxed_sys(&P.rep->state, (P.epoch << 8) | WS_EXITED);
    }
  }
}

}  // namespace gpuos
