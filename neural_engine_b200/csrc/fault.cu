// fault.cu -- host-side fault injection for the callers' failure paths.
//
// The reference has no fault injection (an ANE eval failure is printed,
// io.h:195; a compile failure exits, train.m:298-300).  Here every C-ABI call
// returns a status, and NE_FAULT_INJECT makes chosen calls fail on the host,
// before they do any work: "<entry>:<n>[:<status>]" items, comma-separated,
// fail the n-th call of `entry` with <status>.  Nothing here touches a GPU.
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ne.h"
#include "ne_fault.h"

namespace ne {

namespace {

struct Item {
  std::string entry;
  long long nth;
  ne_status status;
  std::atomic<long long> calls{0};
};

ne_status parse_status(const std::string& s) {
  if (s == "io") return NE_ERR_IO;
  if (s == "format") return NE_ERR_FORMAT;
  if (s == "oom") return NE_ERR_OOM;
  if (s == "timeout") return NE_ERR_TIMEOUT;
  if (s == "state") return NE_ERR_STATE;
  return NE_ERR_CUDA;
}

// Parsed once; malformed items are ignored.
std::vector<Item*>& items() {
  static std::vector<Item*> v = [] {
    std::vector<Item*> out;
    const char* e = std::getenv("NE_FAULT_INJECT");
    if (!e) return out;
    std::string all(e);
    size_t at = 0;
    while (at <= all.size()) {
      size_t end = all.find(',', at);
      if (end == std::string::npos) end = all.size();
      const std::string it = all.substr(at, end - at);
      at = end + 1;
      const size_t c1 = it.find(':');
      if (c1 == std::string::npos || c1 == 0) continue;
      const size_t c2 = it.find(':', c1 + 1);
      const std::string num = it.substr(c1 + 1, c2 == std::string::npos ? std::string::npos
                                                                          : c2 - c1 - 1);
      char* stop = nullptr;
      const long long n = std::strtoll(num.c_str(), &stop, 10);
      if (num.empty() || *stop != '\0' || n < 1) continue;
      Item* x = new Item();   // lives for the process
      x->entry = it.substr(0, c1);
      x->nth = n;
      x->status = c2 == std::string::npos ? NE_ERR_CUDA : parse_status(it.substr(c2 + 1));
      out.push_back(x);
    }
    return out;
  }();
  return v;
}

}  // namespace

bool fault_point(const char* entry, ne_status* status) {
  std::vector<Item*>& v = items();
  if (v.empty()) return false;
  bool hit = false;
  for (Item* x : v) {
    if (x->entry != entry) continue;
    const long long k = x->calls.fetch_add(1) + 1;
    if (k == x->nth && !hit) {
      *status = x->status;
      hit = true;
    }
  }
  return hit;
}

}  // namespace ne

extern "C" NE_API int ne_fault_calls(const char* entry) {
  if (!entry) return 0;
  for (ne::Item* x : ne::items())
    if (x->entry == entry) return (int)x->calls.load();
  return 0;
}
