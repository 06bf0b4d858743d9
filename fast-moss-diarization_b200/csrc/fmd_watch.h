// No-progress detector of the engine's host loop (fmd_engine_step).
//
// The host launches blocks of step graphs and polls the device counters
// between blocks. Every live step emits a token, consumes prompt rows or
// finishes a request, so a run of polls in which none of the three moved
// means the queue cannot make progress (a request that can never be
// admitted, a scheduler stuck on a bad state): the loop then stops with
// FMD_ETIMEDOUT instead of spinning forever. Plain C++, no CUDA, so the
// detector is tested on the host with injected stalls.
#ifndef FMD_WATCH_H
#define FMD_WATCH_H

namespace fmd {

class ProgressWatch {
 public:
  explicit ProgressWatch(int limit) : limit_(limit) {}
  // Feed one poll's counters; true once `limit` consecutive polls saw no
  // change of (tokens + prefill rows + requests done).
  bool stalled(long long gen_tokens, long long prefill_tokens, long long done) {
    const long long progress = gen_tokens + prefill_tokens + done;
    idle_ = progress == last_ ? idle_ + 1 : 0;
    last_ = progress;
    return idle_ >= limit_;
  }
  int idle_polls() const { return idle_; }

 private:
  long long last_ = -1;
  int idle_ = 0;
  int limit_;
};

}  // namespace fmd

#endif  // FMD_WATCH_H
