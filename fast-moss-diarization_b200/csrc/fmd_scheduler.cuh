// On-GPU continuous-batching scheduler state.
#pragma once

#include "fmd_kernels.cuh"

namespace fmd {

enum SlotState { kSlotFree = 0, kSlotPrefill = 1, kSlotDecode = 2 };

// Device copy of one queued request (layout of `fmd_request`).
struct DevRequest {
  int prompt_len;
  int max_new_tokens;
  int forced_stop;
  int reserved;
  long long embed_row;
};

struct DevResult {
  int n_tokens;
  int finish_reason;
};

struct EngineCounters {
  int next_req;        // next queue entry to admit
  int done;            // requests finished
  int free_top;        // entries on the free-page stack
  int status;          // 0 or a negative FMD_E* code
  long long steps;
  long long gen_tokens;
  long long prefill_tokens;
  long long last_kv_tokens;    // sum of (pos + 1) over the decode rows of the latest plan
  long long last_decode_rows;
  long long last_kv_tokens_lo; // the same over decode rows below EngineDev::split_rows
  long long last_rows_lo;
  long long pending_prefill;   // prompt rows admitted but not yet planned
};

struct EngineDev {
  int n_reqs;
  int n_pages;         // pages in the pool
  int consume_only;    // book the previous samples, plan nothing
  int allow_prefill;   // 0: plan decode rows only (decode-only step graph)
  int max_batch;       // slots in use (<= reserved slots)
  int prefill_chunk;   // prompt rows admitted per step
  int max_rows;        // plan capacity R
  int split_rows;      // decode rows below this index run as the first half of a split step (0: no split)
  int max_pages_per_slot;
  int eos;
  int vocab;           // token ids outside [0, vocab) end their request with an error
  int page_tokens;
  int tok_stride;
  const DevRequest* reqs;
  int* slot_state;
  int* slot_req;
  int* slot_len;       // positions cached (or reserved by this step's rows)
  int* slot_pdone;     // prompt rows already planned
  int* slot_ngen;      // tokens emitted
  int* slot_last;      // last emitted token (fed next step)
  int* slot_npages;
  int* free_stack;     // free KV pages
  int* page_table;     // [slots][max_pages_per_slot]
  int* out_tokens;     // [n_reqs][tok_stride]
  DevResult* results;  // [n_reqs]
  EngineCounters* ctr;
  const int* next_ids; // greedy ids of the previous step's sample rows
  Plan plan;
};

void launch_schedule(const EngineDev& e, cudaStream_t s);

}  // namespace fmd
