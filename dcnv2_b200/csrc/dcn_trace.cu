// Kernel timing trace (see dcn_trace.h and dcn_trace_* in include/dcn_b200.h).
#include <mutex>
#include <vector>

#include "dcn_b200.h"
#include "dcn_trace.h"

namespace dcn {

namespace {

const char* kNames[TR_COUNT] = {
    "pack_input",          "pack_weight_fwd",     "forward",
    "pack_weight_bwd",     "zero_accumulators",   "backward_data",
    "backward_weight",     "finish_grad_input",   "finish_grad_weight",
    "pack_grad_output",    "backward_scatter",
};

struct Rec {
  int id;
  cudaEvent_t a, b;
};

std::mutex g_mu;
bool g_on = false;
std::vector<Rec> g_pending;
std::vector<cudaEvent_t> g_pool;
double g_ms[TR_COUNT];
long long g_n[TR_COUNT];

cudaEvent_t get_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

}  // namespace

bool trace_on() { return g_on; }

TraceScope::TraceScope(int id, cudaStream_t s) : id_(id), s_(s), rec_(nullptr) {
  if (!g_on) return;
  std::lock_guard<std::mutex> lk(g_mu);
  Rec* r = new Rec{id, get_event(), get_event()};
  if (r->a && r->b && cudaEventRecord(r->a, s) == cudaSuccess) {
    rec_ = r;
  } else {
    if (r->a) g_pool.push_back(r->a);
    if (r->b) g_pool.push_back(r->b);
    delete r;
  }
}

TraceScope::~TraceScope() {
  if (!rec_) return;
  Rec* r = static_cast<Rec*>(rec_);
  std::lock_guard<std::mutex> lk(g_mu);
  if (cudaEventRecord(r->b, s_) == cudaSuccess) {
    g_pending.push_back(*r);
  } else {
    g_pool.push_back(r->a);
    g_pool.push_back(r->b);
  }
  delete r;
}

}  // namespace dcn

using namespace dcn;

extern "C" {

int dcn_trace_enable(int on) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_on = on != 0;
  return DCN_OK;
}

int dcn_trace_collect(dcn_trace_entry* out, int max_entries) {
  std::lock_guard<std::mutex> lk(g_mu);
  int rc = DCN_OK;
  for (const Rec& r : g_pending) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.b) != cudaSuccess || cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess)
      rc = DCN_E_CUDA;
    g_ms[r.id] += ms;
    g_n[r.id] += 1;
    g_pool.push_back(r.a);
    g_pool.push_back(r.b);
  }
  g_pending.clear();
  if (rc != DCN_OK) return rc;
  int k = 0;
  for (int i = 0; i < TR_COUNT; ++i) {
    if (g_n[i] == 0) continue;
    if (out && k < max_entries) {
      out[k].name = kNames[i];
      out[k].launches = g_n[i];
      out[k].total_ms = g_ms[i];
    }
    ++k;
  }
  return k;
}

int dcn_trace_reset(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (const Rec& r : g_pending) {
    cudaEventSynchronize(r.b);
    g_pool.push_back(r.a);
    g_pool.push_back(r.b);
  }
  g_pending.clear();
  for (int i = 0; i < TR_COUNT; ++i) {
    g_ms[i] = 0.0;
    g_n[i] = 0;
  }
  return DCN_OK;
}

}  // extern "C"
