/* A plain C99 consumer of the library's C ABI (include/csaq_b200.h): the
 * header compiles without C++ and the shared library links and answers
 * host-side calls (identification, sizes, argument validation) with no GPU.
 * Built and run by tests/test_abi_cpu.py. Prints one line per check. */
#include <stddef.h>
#include <stdio.h>
#include <stdint.h>

#include "csaq_b200.h"

int main(void) {
  printf("version %s\n", csaq_version());
  printf("status %s\n", csaq_status_string(CSAQ_ERR_BITS));
  printf("row_bytes %lld %lld %lld %lld\n", (long long)csaq_packed_row_bytes(37, 2),
         (long long)csaq_packed_row_bytes(37, 4), (long long)csaq_packed_row_bytes(37, 8),
         (long long)csaq_packed_row_bytes(37, 16));
  const void* dummy = (const void*)16;
  printf("quant_pack_null %d\n", csaq_quant_pack(NULL, CSAQ_DT_F16, 4, 4, 4, 4, 128, (uint8_t*)16,
                                                  (float*)16, (int32_t*)16, NULL));
  printf("quant_pack_bits %d\n", csaq_quant_pack(dummy, CSAQ_DT_F16, 4, 4, 4, 3, 128, (uint8_t*)16,
                                                  (float*)16, (int32_t*)16, NULL));
  csaq_tier t = {0};
  t.bits = 3;
  t.n_rows = 1;
  t.group_size = 128;
  t.n_groups = 1;
  t.row_bytes = 64;
  printf("qgemv_bits %d\n", csaq_qgemv(&t, 1, 128, dummy, CSAQ_DT_BF16, 1, 128, NULL));
  printf("qgemv_tiers %d\n", csaq_qgemv(&t, 0, 128, dummy, CSAQ_DT_BF16, 1, 128, NULL));
  printf("greedy_null %d\n", csaq_greedy_cliques(NULL, 1, 1, NULL, NULL, NULL));
  int64_t n = -1, site = -1, value = -1, bound = -1;
  printf("checked %d guard %d\n", csaq_checked_build(), csaq_guard_report(&n, &site, &value, &bound));
  /* struct layouts, compared with the Python binding's ctypes mirrors */
  printf("layout_tier %u %u %u %u\n", (unsigned)sizeof(csaq_tier), (unsigned)offsetof(csaq_tier, blocks),
         (unsigned)offsetof(csaq_tier, y), (unsigned)offsetof(csaq_tier, ldr));
  printf("layout_gemv_ext %u %u\n", (unsigned)sizeof(csaq_gemv_ext), (unsigned)offsetof(csaq_gemv_ext, x_mul));
  printf("layout_p2p_group %u %u %u\n", (unsigned)sizeof(csaq_p2p_group), (unsigned)offsetof(csaq_p2p_group, flags),
         (unsigned)offsetof(csaq_p2p_group, err));
  return 0;
}
