/* A plain-C host of the kotflash_b200 C ABI (no Python, no C++): it includes
 * the public header, links against the shared library and exercises the
 * host-side part of the interface that runs without a GPU -- version and
 * workspace queries, and argument checks that must fail before anything is
 * launched.  tests/test_c_host.py compiles it with gcc as C99 and runs it.
 * Exit status 0 means every check held; each failed check prints a line. */
#include <stdio.h>
#include <string.h>

#include "kotflash_b200.h"

static int failures = 0;

static void check(int cond, const char* what) {
  if (!cond) {
    printf("FAILED: %s (last error: %s)\n", what, kf_last_error());
    ++failures;
  }
}

/* a [n0, n1, n2, n3] contiguous view at a fake address: only the host-side
 * checks look at it, nothing is dereferenced */
static kf_tensor4 view(int64_t n0, int64_t n1, int64_t n2, int64_t n3) {
  kf_tensor4 t;
  t.ptr = (void*)0x1000;
  t.size[0] = n0;
  t.size[1] = n1;
  t.size[2] = n2;
  t.size[3] = n3;
  t.stride[3] = 1;
  t.stride[2] = n3;
  t.stride[1] = n2 * n3;
  t.stride[0] = n1 * n2 * n3;
  return t;
}

int main(void) {
  kf_tensor4 kc, vc, nk, nv, q, k, o;
  check(kf_version() >= 10000, "version");
  check(kf_decode_workspace_bytes(2, 8, 1, 64, 1) == 0, "one split needs no workspace");
  check(kf_decode_workspace_bytes(2, 8, 1, 64, 4) >= (size_t)4 * 16 * 65 * 4, "split partials fit");
  check(kf_attn_bwd_workspace_bytes(4, 32, 4096, 128) >= (size_t)4 * 32 * 4096 * 130 * 4,
        "backward workspace holds the dQ accumulator and row statistics");
  check(kf_attn_bwd_workspace_bytes_kv(4, 32, 8, 4096, 4096, 128) >=
            kf_attn_bwd_workspace_bytes(4, 32, 4096, 128),
        "the dK/dV accumulators only add to the backward workspace");
  check(kf_decode_num_splits(2, 8, 2, 1, 131072, 64, 148) >= 2, "long decode is split");
  check(kf_peer_mailbox_bytes(9, 16, 64) == 0, "at most 8 peers");
  check(kf_peer_mailbox_bytes(2, 16, 64) > 0, "mailbox size");

  kc = view(1, 2, 8, 16);
  vc = view(1, 2, 8, 16);
  nk = view(1, 2, 3, 16);
  nv = view(1, 2, 3, 16);
  check(kf_append(&kc, &vc, &nk, &nv, 6, KF_F16, NULL) == KF_ERR_INVALID &&
            strstr(kf_last_error(), "capacity") != NULL,
        "append past the cache capacity is rejected");
  check(kf_append(&kc, &vc, &nk, &nv, 0, 7, NULL) == KF_ERR_INVALID && strstr(kf_last_error(), "dtype") != NULL,
        "unknown dtype is rejected");

  q = view(1, 3, 1, 16);
  k = view(1, 2, 8, 16);
  check(kf_decode(&q, &k, &k, NULL, NULL, 0, &q, NULL, KF_F16, 0.25f, 0, NULL, 0, NULL) == KF_ERR_INVALID &&
            strstr(kf_last_error(), "divisible") != NULL,
        "query heads must be a multiple of the KV heads");
  q = view(1, 4, 17, 16);
  o = view(1, 4, 17, 16);
  check(kf_decode(&q, &k, &k, NULL, NULL, 0, &o, NULL, KF_F16, 0.25f, 0, NULL, 0, NULL) == KF_ERR_UNSUPPORTED,
        "decode takes at most 16 query rows");
  q = view(1, 4, 5, 20);
  k = view(1, 2, 8, 20);
  check(kf_attn_fwd(&q, &k, &k, &q, (float*)0x2000, KF_BF16, 0.2f, 1, NULL, NULL) == KF_ERR_UNSUPPORTED &&
            strstr(kf_last_error(), "multiple of 8") != NULL,
        "head dim must be a multiple of 8");
  check(kf_merge_partials(NULL, NULL, 1, 1, 64, NULL, NULL, KF_F16, NULL) == KF_ERR_INVALID,
        "merge without buffers is rejected");

  if (failures == 0) printf("all C-host checks passed\n");
  return failures == 0 ? 0 : 1;
}
