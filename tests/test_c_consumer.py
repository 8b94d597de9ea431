"""The C ABI from plain C: a C11 program that includes ``include/cruise_epoch.h``
and ``include/cruise_protocol.h`` (no C++ in either), links against the
engine library and calls the entry points that need no GPU -- the presets,
the tensor-parallel shard query, the thread's last create error and the
argument check of the device-prefill bridge call.  This is
what a cgo, JNI or N-API binding compiles against."""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB_DIR = ROOT / "cruise_b200"

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "cruise_epoch.h"
#include "cruise_protocol.h"

int main(void) {
  CruiseModelConfig cfg;
  memset(&cfg, 0, sizeof(cfg));
  if (cruise_epoch_preset("qwen2.5-7b", &cfg) != 0) return 10;
  if (cruise_epoch_preset("no-such-model", &cfg) != -1) return 11;
  if (cruise_epoch_preset("qwen2.5-7b", &cfg) != 0) return 12;
  printf("7b %d %d %d %d %d %d %d %d %d %d\n", cfg.num_layers, cfg.hidden, cfg.num_heads, cfg.num_kv_heads,
         cfg.head_dim, cfg.intermediate, cfg.vocab, cfg.block_size, cfg.blocks_per_row, cfg.num_blocks);
  for (int t = 1; t <= 8; t *= 2) {
    int32_t covered_q = 0, covered_v = 0;
    for (int r = 0; r < t; ++r) {
      int32_t s[8];
      if (cruise_epoch_tp_shard(&cfg, r, t, s) != 0) return 20 + t;
      covered_q += s[1];
      covered_v += s[7];
    }
    printf("tp %d q %d v %d\n", t, covered_q, covered_v);
  }
  int32_t s[8];
  if (cruise_epoch_tp_shard(&cfg, 0, 3, s) != -1) return 30;
  const char *why = cruise_epoch_last_error(NULL);
  printf("last_error %s\n", why == NULL ? "null" : "string");
  /* the device-prefill bridge call rejects a missing handle before any GPU work */
  int64_t tokens[4] = {1, 2, 3, 4};
  int32_t lens[4] = {2, 0, 0, 0};
  if (resident_epoch_prefill(NULL, tokens, lens, 1) != 10) return 40;
  return 0;
}
"""


def test_header_compiles_as_c11_and_links(tmp_path):
    if shutil.which("gcc") is None:
        pytest.skip("gcc not found")
    library = LIB_DIR / "libcruise_epoch.so"
    if not library.exists():
        pytest.skip("engine library not built")
    source = tmp_path / "consumer.c"
    source.write_text(PROGRAM)
    binary = tmp_path / "consumer"
    subprocess.run(
        ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", f"-I{ROOT / 'include'}", str(source),
         "-o", str(binary), f"-L{LIB_DIR}", "-lcruise_epoch", f"-Wl,-rpath,{LIB_DIR}"],
        check=True, capture_output=True, text=True,
    )
    run = subprocess.run([str(binary)], capture_output=True, text=True, timeout=120,
                         env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert run.returncode == 0, (run.returncode, run.stdout, run.stderr)
    lines = run.stdout.splitlines()
    assert lines[0] == "7b 28 3584 28 4 128 18944 152064 128 2 8"
    for t, line in zip((1, 2, 4, 8), lines[1:5]):
        assert line == f"tp {t} q 28 v 152064"
    assert lines[5].startswith("last_error ")
