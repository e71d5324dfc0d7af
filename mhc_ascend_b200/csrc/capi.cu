// Library identification and the per-thread last-error string of the C-ABI.
#include "common.cuh"

#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace mhc {
static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}
}  // namespace mhc

extern "C" const char* mhc_version(void) { return "mhc_ascend_b200 0.1.0 (sm_100a)"; }

extern "C" const char* mhc_get_last_error_string(void) { return mhc::g_last_error; }

namespace mhc {
namespace {
struct ProfRecord {
  const char* name;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRecord> g_prof_records;
std::vector<cudaEvent_t> g_prof_pool;
}  // namespace

bool profiling_enabled() { return g_prof_on; }

cudaEvent_t profile_event() {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

void profile_record(const char* name, cudaEvent_t start, cudaEvent_t stop) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_records.push_back({name, start, stop});
}
}  // namespace mhc

extern "C" int mhc_profile_enable(int enable) {
  std::lock_guard<std::mutex> lk(mhc::g_prof_mu);
  mhc::g_prof_on = enable != 0;
  return MHC_OK;
}

extern "C" int mhc_profile_report(char* buf, size_t cap) {
  std::vector<mhc::ProfRecord> recs;
  {
    std::lock_guard<std::mutex> lk(mhc::g_prof_mu);
    recs.swap(mhc::g_prof_records);
  }
  std::map<std::string, std::pair<long, double>> agg;
  std::vector<std::string> order;
  int rc = MHC_OK;
  for (auto& r : recs) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.stop) != cudaSuccess ||
        cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess) {
      rc = mhc::fail(MHC_ERR_CUDA, "mhc_profile_report: event query failed");
    }
    auto it = agg.find(r.name);
    if (it == agg.end()) {
      order.push_back(r.name);
      agg[r.name] = {1, (double)ms};
    } else {
      it->second.first += 1;
      it->second.second += ms;
    }
  }
  {
    std::lock_guard<std::mutex> lk(mhc::g_prof_mu);
    for (auto& r : recs) {
      mhc::g_prof_pool.push_back(r.start);
      mhc::g_prof_pool.push_back(r.stop);
    }
  }
  if (rc) return rc;
  std::string out;
  for (auto& n : order) {
    char line[256];
    snprintf(line, sizeof(line), "%s %ld %.6f\n", n.c_str(), agg[n].first, agg[n].second);
    out += line;
  }
  if (buf && cap > 0) {
    size_t k = out.size() < cap - 1 ? out.size() : cap - 1;
    memcpy(buf, out.data(), k);
    buf[k] = 0;
  }
  return (int)out.size();
}
