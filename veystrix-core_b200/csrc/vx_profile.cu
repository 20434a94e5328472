// Stage timing: CUDA events recorded on the caller's stream between the
// kernels of one entry-point call (see vx_profile_enable in vxmoe.h).
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "vx_common.cuh"
#include "vx_profile.h"

namespace vx {
namespace {

struct Mark {
  std::string label;   // stage that ends at this event ("" opens a call)
  cudaEvent_t ev;
};

std::mutex g_mu;
bool g_enabled = false;
std::vector<Mark> g_marks;
std::vector<cudaEvent_t> g_free;

cudaEvent_t take_event() {
  if (!g_free.empty()) {
    cudaEvent_t e = g_free.back();
    g_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

}  // namespace

bool profile_on() { return g_enabled; }

void profile_mark(cudaStream_t st, const char* label) {
  if (!g_enabled) return;
  std::lock_guard<std::mutex> lk(g_mu);
  cudaEvent_t e = take_event();
  if (!e) return;
  cudaEventRecord(e, st);
  g_marks.push_back({label ? label : "", e});
}

}  // namespace vx

using namespace vx;

extern "C" int vx_profile_enable(int enabled) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto& m : g_marks) g_free.push_back(m.ev);
  g_marks.clear();
  g_enabled = enabled != 0;
  return VX_OK;
}

extern "C" int vx_profile_read(int max_stages, char* labels, int labels_cap, double* avg_ms,
                               int32_t* counts, int32_t* n_stages) {
  std::lock_guard<std::mutex> lk(g_mu);
  std::vector<std::string> names;
  std::vector<double> sum;
  std::vector<int> cnt;
  if (!g_marks.empty()) {
    cudaError_t e = cudaEventSynchronize(g_marks.back().ev);
    if (e != cudaSuccess) return vx_cuda_fail(e);
  }
  for (size_t i = 1; i < g_marks.size(); ++i) {
    if (g_marks[i].label.empty()) continue;  // a new call starts here
    float ms = 0.f;
    cudaError_t e = cudaEventElapsedTime(&ms, g_marks[i - 1].ev, g_marks[i].ev);
    if (e != cudaSuccess) return vx_cuda_fail(e);
    size_t j = 0;
    while (j < names.size() && names[j] != g_marks[i].label) ++j;
    if (j == names.size()) {
      names.push_back(g_marks[i].label);
      sum.push_back(0.0);
      cnt.push_back(0);
    }
    sum[j] += ms;
    cnt[j] += 1;
  }
  const int n = int(names.size());
  if (n_stages) *n_stages = n;
  std::string joined;
  for (int j = 0; j < n && j < max_stages; ++j) {
    if (avg_ms) avg_ms[j] = cnt[j] ? sum[j] / cnt[j] : 0.0;
    if (counts) counts[j] = cnt[j];
    joined += names[j];
    joined += '\n';
  }
  if (labels && labels_cap > 0) {
    const size_t m = std::min<size_t>(joined.size(), size_t(labels_cap - 1));
    memcpy(labels, joined.data(), m);
    labels[m] = '\0';
  }
  return VX_OK;
}
