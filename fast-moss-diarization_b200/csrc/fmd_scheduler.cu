// On-GPU continuous-batching scheduler.
//
// Replaces the host loop of `Engine::generate_batch` (crates/fmd-core/src/
// engine.rs:505-538) and the static micro-batching of `Engine::transcribe`
// (engine.rs:382-424). One single-CTA kernel runs at the start of every step:
//   1. consume the previous step's greedy ids (EOS / forced end-of-turn /
//      budget -> finish, engine.rs:509-523), freeing the slot's KV pages;
//   2. refill free slots from the device request queue, reserving
//      ceil((prompt + budget) / 64) pages from a device free stack;
//   3. build the next plan: one decode row per decoding slot, then up to
//      `prefill_chunk` prompt rows of prefilling slots (chunked prefill mixed
//      with decode), the sample rows, the prefill attention blocks and the
//      decode split items.
// Nothing waits on the host; the host polls `EngineCounters` every few steps.
// All loops are bounded by the slot / row capacities.
#include "fmd_scheduler.cuh"

namespace fmd {

namespace {

constexpr int kMaxSlots = 256;
constexpr int kFinishStop = 0, kFinishLength = 1, kFinishError = 2;
constexpr int kStatusNoMem = -12;
constexpr int kStatusBadToken = -5;  // FMD_EIO

__global__ void __launch_bounds__(256) k_schedule(EngineDev e) {
  __shared__ int s_seg_row0[kMaxSlots], s_seg_n[kMaxSlots], s_seg_pos0[kMaxSlots], s_seg_item0[kMaxSlots];
  __shared__ long long s_seg_emb0[kMaxSlots];
  __shared__ int s_seg_sample[kMaxSlots];
  __shared__ int s_n_rows, s_n_decode, s_n_sample, s_n_pblocks, s_n_items, s_finished;
  // shared copies of the slot state: every global array is read once, in
  // parallel, so the serial bookkeeping below runs on shared memory
  __shared__ int st_state[kMaxSlots], st_req[kMaxSlots], st_len[kMaxSlots], st_pdone[kMaxSlots],
      st_ngen[kMaxSlots], st_last[kMaxSlots], st_npages[kMaxSlots];
  __shared__ DevRequest st_rq[kMaxSlots];  // request of each occupied slot
  __shared__ int smp_slot[kMaxSlots], smp_tok[kMaxSlots];
  __shared__ EngineCounters s_ctr;
  __shared__ int s_prev;
  // page moves recorded by the serial bookkeeping and done by all threads:
  // the pages of finished slots onto the free stack (frees) and off it into
  // admitted slots' page tables (allocations), in the stack's LIFO order
  __shared__ int s_nf, fin_slot[kMaxSlots], fin_np[kMaxSlots], fin_base[kMaxSlots];
  __shared__ int s_na, adm_slot[kMaxSlots], adm_need[kMaxSlots], adm_top[kMaxSlots];
  PlanCounts* cnt = e.plan.counts;
  const int nb = e.max_batch;

  if (threadIdx.x == 0) {
    s_ctr = *e.ctr;
    s_prev = cnt->n_sample;
  }
  for (int s = threadIdx.x; s < nb; s += blockDim.x) {
    st_state[s] = e.slot_state[s];
    st_req[s] = e.slot_req[s];
    st_len[s] = e.slot_len[s];
    st_pdone[s] = e.slot_pdone[s];
    st_ngen[s] = e.slot_ngen[s];
    st_last[s] = e.slot_last[s];
    st_npages[s] = e.slot_npages[s];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < s_prev; i += blockDim.x) {
    smp_slot[i] = e.plan.sample_slot[i];
    smp_tok[i] = e.next_ids[i];
  }
  for (int s = threadIdx.x; s < nb; s += blockDim.x)
    if (st_state[s] != kSlotFree) st_rq[s] = e.reqs[st_req[s]];
  __syncthreads();

  if (threadIdx.x == 0) {
    EngineCounters* c = &s_ctr;
    // ---- 1. consume the previous step's samples ----
    const int prev = s_prev;
    long long emitted = 0;
    int nf = 0;
    for (int i = 0; i < prev; ++i) {
      const int slot = smp_slot[i];
      const int tok = smp_tok[i];
      if (st_state[slot] == kSlotFree) continue;
      const int req = st_req[slot];
      const DevRequest rq = st_rq[slot];
      const int ng = st_ngen[slot];
      int finish = -1;
      if (rq.max_new_tokens <= 0) {
        finish = kFinishLength;
      } else if (tok < 0 || tok >= e.vocab) {
        // never fed back: an id outside the vocabulary would index past the
        // embedding table (the greedy pick has already flagged the step)
        finish = kFinishError;
        c->status = kStatusBadToken;
      } else if (tok == e.eos || (rq.forced_stop >= 0 && ng == rq.forced_stop)) {
        finish = kFinishStop;
      } else {
        e.out_tokens[(size_t)req * e.tok_stride + ng] = tok;
        st_ngen[slot] = ng + 1;
        st_last[slot] = tok;
        st_state[slot] = kSlotDecode;
        ++emitted;
        if (ng + 1 >= rq.max_new_tokens) finish = kFinishLength;
      }
      if (finish >= 0) {
        e.results[req].n_tokens = st_ngen[slot];
        e.results[req].finish_reason = finish;
        // its pages go onto the free stack at free_top .. free_top + np - 1
        fin_slot[nf] = slot;
        fin_np[nf] = st_npages[slot];
        fin_base[nf] = c->free_top;
        c->free_top += st_npages[slot];
        ++nf;
        st_npages[slot] = 0;
        st_state[slot] = kSlotFree;
        c->done += 1;
      }
    }
    c->gen_tokens += emitted;
    s_nf = nf;
    s_na = 0;
    if (e.consume_only) {
      cnt->n_rows = cnt->n_decode = cnt->n_sample = cnt->n_pblocks = cnt->n_ditems = 0;
      cnt->finished = c->done >= e.n_reqs ? 1 : 0;
    }
  }
  __syncthreads();
  for (int f = 0; f < s_nf; ++f) {
    const int* pt = e.page_table + (size_t)fin_slot[f] * e.max_pages_per_slot;
    for (int k = threadIdx.x; k < fin_np[f]; k += blockDim.x) e.free_stack[fin_base[f] + k] = pt[k];
  }
  __syncthreads();  // the freed pages are on the stack before admission pops them
  if (!e.consume_only && threadIdx.x == 0) {
    EngineCounters* c = &s_ctr;

    // ---- 2. admit queued requests into free slots ----
    int na = 0;
    for (int s = 0; s < nb && c->next_req < e.n_reqs; ++s) {
      if (st_state[s] != kSlotFree) continue;
      const DevRequest rq = e.reqs[c->next_req];
      const int budget = rq.max_new_tokens > 0 ? rq.max_new_tokens : 0;
      const int need = (rq.prompt_len + budget + e.page_tokens - 1) / e.page_tokens;
      if (rq.prompt_len <= 0 || need > e.max_pages_per_slot || need > e.n_pages) {
        // can never be served: fail this request alone (engine.rs:414-421)
        e.results[c->next_req].n_tokens = 0;
        e.results[c->next_req].finish_reason = kFinishError;
        c->done += 1;
        c->status = kStatusNoMem;
        c->next_req += 1;
        --s;
        continue;
      }
      if (need > c->free_top) break;  // wait for pages to come back (FIFO)
      // page k of the slot is stack entry free_top - 1 - k
      adm_slot[na] = s;
      adm_need[na] = need;
      adm_top[na] = c->free_top;
      c->free_top -= need;
      ++na;
      st_npages[s] = need;
      st_state[s] = kSlotPrefill;
      st_req[s] = c->next_req;
      st_rq[s] = rq;
      st_len[s] = 0;
      st_pdone[s] = 0;
      st_ngen[s] = 0;
      c->next_req += 1;
    }
    s_na = na;

    // ---- 3. lay out the next plan (segment descriptors) ----
    int rows = 0, items = 0, samples = 0, pblocks = 0;
    long long kv_tokens = 0, kv_lo = 0;
    for (int s = 0; s < nb; ++s) {
      s_seg_n[s] = 0;
      if (st_state[s] == kSlotDecode && rows < e.max_rows) {
        kv_tokens += st_len[s] + 1;
        if (rows < e.split_rows) kv_lo += st_len[s] + 1;
        s_seg_row0[s] = rows;
        s_seg_n[s] = 1;
        s_seg_pos0[s] = st_len[s];
        s_seg_item0[s] = items;
        s_seg_sample[s] = samples;
        st_len[s] += 1;
        items += (st_len[s] + kDecodeItemTokens - 1) / kDecodeItemTokens;
        rows += 1;
        samples += 1;
      }
    }
    const int n_decode = rows;
    c->last_kv_tokens = kv_tokens;
    c->last_decode_rows = n_decode;
    c->last_kv_tokens_lo = kv_lo;
    c->last_rows_lo = n_decode < e.split_rows ? n_decode : e.split_rows;
    int budget_rows = e.allow_prefill ? e.prefill_chunk : 0;
    long long pending = 0;
    for (int s = 0; s < nb; ++s) {
      if (st_state[s] != kSlotPrefill) continue;
      const DevRequest rq = st_rq[s];
      pending += rq.prompt_len - st_pdone[s];
      const int left = rq.prompt_len - st_pdone[s];
      int take = left < budget_rows ? left : budget_rows;
      if (take > e.max_rows - rows) take = e.max_rows - rows;
      if (take <= 0) continue;
      s_seg_row0[s] = rows;
      s_seg_n[s] = take;
      s_seg_pos0[s] = st_len[s];
      s_seg_emb0[s] = rq.embed_row + st_pdone[s];
      s_seg_item0[s] = pblocks;
      s_seg_sample[s] = take == left ? samples++ : -1;
      st_pdone[s] += take;
      st_len[s] += take;
      rows += take;
      pblocks += (take + kRowsPerPBlock - 1) / kRowsPerPBlock;
      budget_rows -= take;
      c->prefill_tokens += take;
      pending -= take;
    }
    c->pending_prefill = pending;
    s_n_rows = rows;
    s_n_decode = n_decode;
    s_n_sample = samples;
    s_n_pblocks = pblocks;
    s_n_items = items;
    s_finished = c->done >= e.n_reqs ? 1 : 0;
    if (rows > 0) c->steps += 1;
  }
  __syncthreads();
  for (int a = 0; a < s_na; ++a) {
    int* pt = e.page_table + (size_t)adm_slot[a] * e.max_pages_per_slot;
    for (int k = threadIdx.x; k < adm_need[a]; k += blockDim.x) pt[k] = e.free_stack[adm_top[a] - 1 - k];
  }
  // ---- write the slot state and counters back ----
  for (int s = threadIdx.x; s < nb; s += blockDim.x) {
    e.slot_state[s] = st_state[s];
    e.slot_req[s] = st_req[s];
    e.slot_len[s] = st_len[s];
    e.slot_pdone[s] = st_pdone[s];
    e.slot_ngen[s] = st_ngen[s];
    e.slot_last[s] = st_last[s];
    e.slot_npages[s] = st_npages[s];
  }
  if (threadIdx.x == 0) *e.ctr = s_ctr;
  if (e.consume_only) return;

  // ---- 4. fill the plan arrays in parallel ----
  for (int s = 0; s < e.max_batch; ++s) {
    const int n = s_seg_n[s];
    if (n == 0) continue;
    const int row0 = s_seg_row0[s], pos0 = s_seg_pos0[s];
    const bool dec = row0 < s_n_decode;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int r = row0 + i;
      e.plan.row_slot[r] = s;
      e.plan.row_pos[r] = pos0 + i;
      e.plan.row_tok[r] = dec ? st_last[s] : -1;
      e.plan.row_emb[r] = dec ? 0 : (int)(s_seg_emb0[s] + i);
    }
    if (dec) {
      const int kv_len = pos0 + 1;
      const int it0 = s_seg_item0[s];
      const int nit = (kv_len + kDecodeItemTokens - 1) / kDecodeItemTokens;
      for (int j = threadIdx.x; j < nit; j += blockDim.x) {
        e.plan.di_row[it0 + j] = row0;
        e.plan.di_start[it0 + j] = j * kDecodeItemTokens;
        e.plan.di_end[it0 + j] = min(kv_len, (j + 1) * kDecodeItemTokens);
      }
      if (threadIdx.x == 0) {
        e.plan.drow_item0[row0] = it0;
        e.plan.drow_nitems[row0] = nit;
        e.plan.sample_row[s_seg_sample[s]] = row0;
        e.plan.sample_slot[s_seg_sample[s]] = s;
      }
    } else {
      const int pb0 = s_seg_item0[s];
      const int nb = (n + kRowsPerPBlock - 1) / kRowsPerPBlock;
      for (int j = threadIdx.x; j < nb; j += blockDim.x) {
        e.plan.pb_row0[pb0 + j] = row0 + j * kRowsPerPBlock;
        e.plan.pb_n[pb0 + j] = min(kRowsPerPBlock, n - j * kRowsPerPBlock);
      }
      if (threadIdx.x == 0 && s_seg_sample[s] >= 0) {
        e.plan.sample_row[s_seg_sample[s]] = row0 + n - 1;
        e.plan.sample_slot[s_seg_sample[s]] = s;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    cnt->n_rows = s_n_rows;
    cnt->n_decode = s_n_decode;
    cnt->n_sample = s_n_sample;
    cnt->n_pblocks = s_n_pblocks;
    cnt->n_ditems = s_n_items;
    cnt->finished = s_finished;
  }
}

}  // namespace

void launch_schedule(const EngineDev& e, cudaStream_t s) { k_schedule<<<1, 256, 0, s>>>(e); }

}  // namespace fmd
