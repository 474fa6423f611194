// TEST INFRASTRUCTURE ONLY: writes the reference's attention-policy gather
// table (src/nn/tables/attention_policy_map.h:15, 64*64 + 8*24 entries of
// int16) to a binary file so the golden fixture can pin our own generated
// table against it.
#include "nn/tables/attention_policy_map.h"
#include <cstdio>
int main(int argc, char **argv) {
  if (argc != 2) return 2;
  std::FILE *f = std::fopen(argv[1], "wb");
  if (!f) return 1;
  const auto &t = MetalFish::NN::Tables::kAttnPolicyMap;
  const bool ok = std::fwrite(t, sizeof(t[0]), sizeof(t) / sizeof(t[0]), f) == sizeof(t) / sizeof(t[0]);
  std::fclose(f);
  return ok ? 0 : 1;
}
