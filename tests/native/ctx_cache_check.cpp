// CPU check of walsh::ContextAddressCache (the per-context address cache of
// the allocation-free entry points).  Exit status 0 when every check passes.
#include <cstdio>
#include <cstdint>

#include "ctx_cache.h"

static int failures = 0;
#define CHECK(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::printf("FAILED line %d: %s\n", __LINE__, #c);           \
      ++failures;                                                  \
    }                                                              \
  } while (0)

int main() {
  int a, b, c, d;
  walsh::ContextAddressCache<3> cache;
  // id 0 means "no context": never cached, never found
  cache.insert(0, &a);
  CHECK(cache.find(0) == nullptr);
  CHECK(cache.size() == 0);
  // a context's first lookup misses, later ones hit
  CHECK(cache.find(11) == nullptr);
  cache.insert(11, &a);
  CHECK(cache.find(11) == &a);
  // a new context on the same device (after a reset: a new, never reused id)
  // misses although the device number is the same
  CHECK(cache.find(12) == nullptr);
  cache.insert(12, &b);
  CHECK(cache.find(12) == &b);
  CHECK(cache.find(11) == &a);
  // re-inserting an id replaces its address and takes no new slot
  cache.insert(12, &c);
  CHECK(cache.find(12) == &c);
  CHECK(cache.size() == 2);
  // a null address is never stored
  cache.insert(13, nullptr);
  CHECK(cache.find(13) == nullptr);
  // full table: the oldest entry is evicted first
  cache.insert(13, &c);
  cache.insert(14, &d);
  CHECK(cache.size() == 3);
  CHECK(cache.find(11) == nullptr);
  CHECK(cache.find(12) == &c);
  CHECK(cache.find(13) == &c);
  CHECK(cache.find(14) == &d);
  cache.insert(15, &a);
  CHECK(cache.find(12) == nullptr);
  CHECK(cache.find(15) == &a);
  if (failures == 0) std::printf("ctx_cache ok\n");
  return failures == 0 ? 0 : 1;
}
