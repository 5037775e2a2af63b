/* A C program that builds a two-tile profile report through include/ipug.h
 * alone (ipug_profile_encode; no GPU calls) and writes the Cap'n Proto bytes
 * to the file named by argv[1].  tests/test_headers_c.py decodes it. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "ipug.h"

int main(int argc, char **argv) {
  if (argc != 2) return 2;
  const char *meta0[] = {"operations", "0,1", "tflops", "1450.5"};
  const ipug_exchange_activity acts[] = {{0u, 10u, 20u}, {2u, 5u, 6u}};
  ipug_profile_sample s0[2] = {
      {0u, 0u, 0u, IPUG_STEP_COMPUTE, "operation.0", "gemm_f16+gelu", meta0, 2u, NULL, 0u, 0u, 0u, 1000u},
      {1u, 1u, 0u, IPUG_STEP_EXCHANGE, "operation.1", NULL, NULL, 0u, acts, 2u, 77u, 1000u, 1500u},
  };
  ipug_profile_sample s1[1] = {
      {0u, 0u, 2u, IPUG_STEP_IDLE, NULL, "k", NULL, 0u, NULL, 0u, 0u, 7u, 9u},
  };
  const ipug_profile_tile tiles[2] = {{3u, s0, 2u}, {4u, s1, 1u}};
  uint64_t need = 0;
  if (ipug_profile_encode(1000000000ull, tiles, 2u, NULL, 0u, &need) != IPUC_ERR_INVALID_ARGUMENT) return 3;
  void *buf = malloc(need);
  if (!buf) return 4;
  if (ipug_profile_encode(1000000000ull, tiles, 2u, buf, need, &need) != IPUC_OK) return 5;
  /* an out-of-range step kind is rejected */
  s1[0].kind = 9u;
  uint64_t scratch = 0;
  if (ipug_profile_encode(1u, tiles, 2u, NULL, 0u, &scratch) != IPUC_ERR_INVALID_ARGUMENT) return 6;
  FILE *f = fopen(argv[1], "wb");
  if (!f) return 7;
  const size_t wrote = fwrite(buf, 1, (size_t)need, f);
  fclose(f);
  free(buf);
  return wrote == need ? 0 : 8;
}
