"""The C ABI from a plain C host, no GPU and no Python in the loop: the public header
compiles as strict C99 and as C++, a C program links the built library and plans a mixed
step with pa_plan_step (the host-only part of the per-step call sequence), and its packed
metadata is word-for-word what the Python binding produces for the same batch; a contract
violation returns PA_ERR_INVALID_ARGUMENT with the reference's message
(inference_server/core/attention.py:202-219)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]

C_HOST = r"""
#include <stdio.h>
#include <stdlib.h>
#include "paged_attention_b200.h"

int main(void) {
  /* one decode sequence (context 20, blocks 7 and 3) and one 5-token prefill (block 9) */
  const int64_t ctx[2] = {20, 5};
  const int64_t ql[2] = {1, 5};
  const int64_t tables[2][4] = {{7, 3, 0, 0}, {9, 0, 0, 0}};
  const int64_t bad_ql[2] = {1, 6};
  pa_step_plan plan;
  int32_t* meta;
  int64_t t, cap;
  int32_t rc;

  /* size query: no buffer, capacity 0 */
  rc = pa_plan_step(ctx, ql, 2, &tables[0][0], 4, 4, 6, 16, 16, 2, 148, 0, NULL, 0, &plan);
  if (rc != PA_OK) { printf("size query failed: %s\n", pa_last_error()); return 1; }
  cap = plan.words;
  meta = (int32_t*)malloc((size_t)cap * sizeof(int32_t));
  rc = pa_plan_step(ctx, ql, 2, &tables[0][0], 4, 4, 6, 16, 16, 2, 148, 0, meta, cap, &plan);
  if (rc != PA_OK) { printf("plan failed: %s\n", pa_last_error()); return 1; }
  printf("abi %d\n", pa_abi_version());
  printf("plan %d %d %d %d\n", plan.num_tokens, plan.num_decode_seqs, plan.num_prefill_seqs, plan.table_width);
  printf("words");
  for (t = 0; t < plan.words; ++t) printf(" %d", meta[t]);
  printf("\n");
  rc = pa_plan_step(ctx, bad_ql, 2, &tables[0][0], 4, 4, 7, 16, 16, 2, 148, 0, meta, cap, &plan);
  printf("bad %d %s\n", rc, pa_last_error());
  free(meta);
  return 0;
}
"""


def _lib_dir(pkg) -> Path:
    return Path(pkg._lib.LIB_PATH).parent


@pytest.mark.skipif(shutil.which("gcc") is None or shutil.which("g++") is None, reason="needs gcc and g++")
def test_c_host_plans_the_same_step_as_the_python_binding(pkg, tmp_path):
    pkg._lib.lib()                                       # builds nothing; the library must exist
    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    inc = str(ROOT / "include")
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-x", "c++", "-I", inc,
                    str(src)], check=True)
    exe = tmp_path / "host"
    lib_dir = str(_lib_dir(pkg))
    subprocess.run(["gcc", "-std=c99", "-pedantic", "-Wall", "-Wextra", "-Werror", "-I", inc, str(src), "-o", str(exe),
                    "-L", lib_dir, "-lpaged_attn_b200", f"-Wl,-rpath,{lib_dir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines()

    assert out[0] == f"abi {pkg._lib.ABI_VERSION}"
    assert out[1] == "plan 6 1 1 2"                     # 6 tokens, 1 decode + 1 prefill sequence, width 2
    words = np.array([int(x) for x in out[2].split()[1:]], dtype=np.int32)
    meta = pkg.StepMetadata.plan_host(np.array([20, 5]), np.array([1, 5]), np.array([[7, 3, 0, 0], [9, 0, 0, 0]]),
                                      num_tokens=6, pool_num_blocks=16, block_size=16, num_kv_heads=2, sm=148)
    np.testing.assert_array_equal(words, meta.host[:int(meta.plan.words)])
    off = int(meta.plan.off_slot_mapping)
    assert words[off:off + 6].tolist() == [3 * 16 + 3, 144, 145, 146, 147, 148]   # position 19 -> block 3
    assert out[3].startswith("bad 1 ") and "query_len exceeds context_len" in out[3]
