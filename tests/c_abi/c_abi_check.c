/* A C (not C++) program against the library's boundary: include/fa4cp_b200.h compiles as
 * C, the library links, and the host-only entry points answer without a GPU:
 * fa4cp_version, argument validation (FA4CP_ERR_INVALID with its text), the copy-engine
 * ring plan and the kv8 workspace size.  Built and run by tests/test_capi.py. */
#include <stdio.h>
#include <string.h>

#include "fa4cp_b200.h"

int main(void) {
  if (fa4cp_version() < 100) return 1;
  /* bad argument: at least one state is required */
  if (fa4cp_merge_states(NULL, NULL, 0, NULL, NULL, 1, 1, 8, FA4CP_DTYPE_BF16, NULL) !=
      FA4CP_ERR_INVALID)
    return 2;
  if (strstr(fa4cp_last_error(), "num_states") == NULL) return 3;
  /* the plan of a 4-rank copy-engine ring call, host only */
  fa4cp_ring_op ops[256];
  const int n = fa4cp_ring_ce_plan(4, 1, 0, 1, ops, 256);
  if (n <= 0) return 4;
  int fused = 0, copies = 0;
  for (int i = 0; i < n; ++i) {
    fused += ops[i].kind == FA4CP_RING_OP_ATTN_FUSED;
    copies += ops[i].kind == FA4CP_RING_OP_COPY;
  }
  if (fused != 1 || copies != 6) return 5;
  if (fa4cp_attn_kv8_workspace_bytes(1024, 2, 128) != 2LL * 1024 * 2 * 128 * 2) return 6;
  printf("c abi ok: version %d, %d plan ops\n", fa4cp_version(), n);
  return 0;
}
