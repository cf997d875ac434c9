"""Layout of the NVLink peer buffer (forgeml_b200/csrc/peer_layout.cuh), checked
on the CPU: the header is compiled with g++ into a small program that prints
every region's byte ranges, and the test asserts that the GEMM-epilogue
exchange, the LL and the two-shot LL all-reduce regions (data sets, flags,
epochs) are pairwise disjoint, aligned as their kernels access them, and
inside the allocation neb_ar_create makes (Layout::total)."""

import shutil
import subprocess
from pathlib import Path

import pytest

HEADER = Path(__file__).resolve().parent.parent / "forgeml_b200" / "csrc" / "peer_layout.cuh"

PROGRAM = r"""
#define __host__
#define __device__
#define __forceinline__ inline
#include <cstdio>
#include "peer_layout.cuh"
using fml::peer::Layout;
int main(int argc, char** argv) {
  Layout l;
  l.slot_bytes = atoll(argv[1]);
  l.world = atoi(argv[2]);
  l.nsub = (int)((l.slot_bytes + 1023) / 1024);
  printf("total %lld\n", l.total());
  for (int set = 0; set < 2; ++set)
    for (int s = 0; s < l.world; ++s) printf("data %lld %lld\n", l.ex_data_off(set, s), l.slot_bytes);
  for (int set = 0; set < 2; ++set)
    for (int s = 0; s < l.world; ++s) printf("flags %lld %lld\n", l.ex_flag_off(set, s, 0), (long long)l.nsub * 4);
  printf("epochs %lld %lld\n", l.ex_epoch_off(0), (long long)l.nsub * 4);
  for (int set = 0; set < 2; ++set)
    for (int s = 0; s < l.world; ++s) printf("lldata %lld %lld\n", l.ll_data_off(set, s), 2 * l.slot_bytes);
  printf("llepochs %lld %lld\n", l.ll_epoch_off(0), (long long)fml::peer::kArBlocks * 4);
  for (int set = 0; set < 2; ++set)
    for (int s = 0; s < l.world; ++s) printf("tsrs %lld %lld\n", l.ts_rs_off(set, s), 2 * l.slot_bytes);
  for (int set = 0; set < 2; ++set) printf("tsag %lld %lld\n", l.ts_ag_off(set), 2 * l.slot_bytes);
  printf("tsepochs %lld %lld\n", l.ts_epoch_off(0), (long long)fml::peer::kArBlocks * 4);
  return 0;
}
"""


@pytest.fixture(scope="module")
def layout_bin(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    d = tmp_path_factory.mktemp("peer_layout")
    src = d / "layout.cpp"
    src.write_text(PROGRAM.replace("#include <cstdio>", "#include <cstdio>\n#include <cstdlib>"))
    exe = d / "layout"
    subprocess.run([gxx, "-std=c++17", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    return exe


@pytest.mark.parametrize("slot_bytes,world", [(131072, 2), (131072, 8), (524288, 4), (16384, 2), (2048 * 64, 1)])
def test_regions_disjoint_and_inside_the_buffer(layout_bin, slot_bytes, world):
    out = subprocess.run([str(layout_bin), str(slot_bytes), str(world)], check=True, capture_output=True,
                         text=True).stdout.split("\n")
    total = int(out[0].split()[1])
    spans = []
    for line in out[1:]:
        if not line.strip():
            continue
        name, off, size = line.split()
        off, size = int(off), int(size)
        assert off >= 0 and off + size <= total, (name, off, size, total)
        # data slots are read and written with 16-byte vectors, flags/epochs as u32
        assert off % (16 if name.startswith(("data", "lldata", "tsrs", "tsag")) else 4) == 0, (name, off)
        spans.append((off, off + size, name))
    spans.sort()
    for (a0, a1, an), (b0, b1, bn) in zip(spans, spans[1:]):
        assert a1 <= b0, f"{an} [{a0},{a1}) overlaps {bn} [{b0},{b1})"
