// The check build's reporting: every translation unit compiled with -DRLENV_CHECKS registers
// a reader of its device check word (common.cuh) when the library loads, and
// rlenv_checks_status ORs them. In the normal build nothing registers, and the entry point
// answers RLENV_EUNSUPPORTED without touching the GPU.
#include <mutex>
#include <vector>

#include "rlenv.h"

namespace rlenv {
namespace {
using Reader = int (*)(unsigned int*, bool);
std::mutex& readers_mutex() {
  static std::mutex m;
  return m;
}
std::vector<Reader>& readers() {
  static std::vector<Reader> v;
  return v;
}
}  // namespace

void register_check_reader(int (*reader)(unsigned int*, bool)) {
  std::lock_guard<std::mutex> lock(readers_mutex());
  readers().push_back(reader);
}

}  // namespace rlenv

extern "C" {

int rlenv_checks_status(unsigned int* word, int clear) {
  using namespace rlenv;
  if (!word) return RLENV_EINVAL;
  *word = 0;
  std::lock_guard<std::mutex> lock(readers_mutex());
  if (readers().empty()) return RLENV_EUNSUPPORTED;
  for (Reader r : readers()) {
    unsigned int w = 0;
    if (int rc = r(&w, clear != 0)) return rc;
    *word |= w;
  }
  return RLENV_OK;
}

}  // extern "C"
