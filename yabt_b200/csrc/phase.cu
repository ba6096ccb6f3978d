// Per-phase device timing and NVTX ranges.
//
// Every launch group of the library sits inside a PhaseScope. The scope
// always opens an NVTX range named after its phase (free when no profiler is
// attached: the NVTX v3 headers only forward to an injected tool). When phase
// timing is on (yabt_phase_timing), the scope also records a CUDA event pair
// on the launching stream from a pool created when timing was switched on;
// yabt_phase_read sums each phase's event intervals. The reference has no
// counterpart (its boosting loop only prints progress, yabt/boosting.py:329-342).
//
// The pool belongs to the device that was current when timing was switched
// on; scopes on other devices are not timed. Timing adds one event record per
// scope boundary, so measure phases in a pass of their own, not inside a timed
// region.
#include <cstdlib>
#include <mutex>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "common.cuh"
#include "../../include/yabt_b200.h"

namespace yabt {

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("YABT_NO_PDL");
    return !(v && v[0] && v[0] != '0');
  }();
  return on;
}

namespace {
thread_local bool t_capturing_level_loop = false;
}
bool capturing_level_loop() { return t_capturing_level_loop; }
void set_capturing_level_loop(bool on) { t_capturing_level_loop = on; }

static const char* const kPhaseNames[PH_COUNT] = {
    "begin", "hist", "reduce", "exchange", "scan", "finalize", "partition", "plan",
    "finish", "leafnet", "interaction", "update", "binning", "collective", "other"};

namespace {
struct PhasePool {
  std::mutex mu;
  bool on = false;
  int device = -1;
  std::vector<cudaEvent_t> ev;   // 2 per range
  std::vector<int> phase;        // phase of each range
  int used = 0;
};
PhasePool& pool() {
  static PhasePool p;
  return p;
}
}  // namespace

bool phase_timing_on() {
  PhasePool& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  return p.on;
}

PhaseScope::PhaseScope(int ph, cudaStream_t s) : slot_(-1), s_(s) {
  nvtxRangePushA(kPhaseNames[ph < 0 || ph >= PH_COUNT ? PH_OTHER : ph]);
  if (capturing_level_loop()) return;        // no event nodes inside a graph loop
  PhasePool& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (!p.on || p.used >= (int)p.phase.size()) return;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != p.device) return;
  slot_ = p.used++;
  p.phase[slot_] = ph;
  cudaEventRecord(p.ev[2 * slot_], s_);
}

PhaseScope::~PhaseScope() {
  if (slot_ >= 0) cudaEventRecord(pool().ev[2 * slot_ + 1], s_);
  nvtxRangePop();
}

}  // namespace yabt

using namespace yabt;

namespace {
// host code brackets its own work (collectives) with push / pop
thread_local std::vector<PhaseScope*> t_host_scopes;
}

extern "C" {

int yabt_phase_count(void) { return PH_COUNT; }

int yabt_phase_name(int phase, char* buf, int len) {
  if (phase < 0 || phase >= PH_COUNT || !buf || len <= 0) { set_error("yabt_phase_name: bad arguments"); return YABT_ERR_ARG; }
  snprintf(buf, (size_t)len, "%s", kPhaseNames[phase]);
  return YABT_OK;
}

int yabt_phase_timing(int max_ranges) {
  PhasePool& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (max_ranges < 0) { set_error("yabt_phase_timing: max_ranges < 0"); return YABT_ERR_ARG; }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) { set_error("yabt_phase_timing: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  if (max_ranges == 0) { p.on = false; return YABT_OK; }
  if (dev != p.device || (int)p.phase.size() < max_ranges) {
    if (p.device >= 0) {
      int cur = dev;
      cudaSetDevice(p.device);
      for (cudaEvent_t ev : p.ev) cudaEventDestroy(ev);
      cudaSetDevice(cur);
    }
    p.ev.assign(2 * (size_t)max_ranges, nullptr);
    for (auto& ev : p.ev) {
      e = cudaEventCreate(&ev);
      if (e != cudaSuccess) {
        set_error("yabt_phase_timing: %s", cudaGetErrorString(e));
        p.ev.clear(); p.phase.clear(); p.device = -1; p.on = false;
        return YABT_ERR_CUDA;
      }
    }
    p.phase.assign((size_t)max_ranges, 0);
    p.device = dev;
  }
  p.used = 0;
  p.on = true;
  return YABT_OK;
}

int yabt_phase_read(double* ms, long long* counts, int nphases) {
  if (!ms || !counts || nphases < PH_COUNT) { set_error("yabt_phase_read: needs %d entries", (int)PH_COUNT); return YABT_ERR_ARG; }
  PhasePool& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  for (int i = 0; i < nphases; ++i) { ms[i] = 0.0; counts[i] = 0; }
  for (int r = 0; r < p.used; ++r) {
    cudaError_t e = cudaEventSynchronize(p.ev[2 * r + 1]);
    float t = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, p.ev[2 * r], p.ev[2 * r + 1]);
    if (e != cudaSuccess) { set_error("yabt_phase_read: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
    ms[p.phase[r]] += t;
    counts[p.phase[r]] += 1;
  }
  return YABT_OK;
}

int yabt_phase_push(int phase, void* stream) {
  if (phase < 0 || phase >= PH_COUNT) { set_error("yabt_phase_push: bad phase"); return YABT_ERR_ARG; }
  t_host_scopes.push_back(new PhaseScope(phase, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_phase_pop(void) {
  if (t_host_scopes.empty()) { set_error("yabt_phase_pop: no open range"); return YABT_ERR_ARG; }
  delete t_host_scopes.back();
  t_host_scopes.pop_back();
  return YABT_OK;
}

}  // extern "C"
