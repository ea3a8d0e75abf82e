// Known-answer vectors for the request-local MT19937 stream (sampling.rs:10-42 of
// the reference): std::mt19937 uses the same init_genrand seeding recurrence and the
// same twist/temper, so its output is an independent statement of the stream.
#include <cstdio>
#include <cstdint>
#include <random>
int main() {
  const uint64_t seeds[] = {0ull, 1ull, 5489ull, 831001ull, 4294967295ull, (1ull << 40) + 7ull};
  printf("{\n");
  for (size_t s = 0; s < sizeof(seeds) / sizeof(seeds[0]); ++s) {
    std::mt19937 g((uint32_t)seeds[s]);  // Generator::new truncates the seed to u32
    printf("  \"%llu\": [", (unsigned long long)seeds[s]);
    for (int i = 0; i < 2000; ++i) printf("%s%u", i ? ", " : "", (unsigned)g());
    printf("]%s\n", s + 1 < sizeof(seeds) / sizeof(seeds[0]) ? "," : "");
  }
  printf("}\n");
  return 0;
}
