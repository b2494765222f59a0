"""Host-side check (CPU, no GPU) of the streamed context-parallel K/V
addressing in csrc/attention_peers.cuh: a small host program built with nvcc
against that header calls ``kv_owner_row`` (the owner rank and local row of
every natural key position, both splits) and ``make_kv_peer_maps`` with a
stub tensor-map encoder that records its arguments instead of encoding.
Both are compared with an independent restatement here: the owner layout of
the zig-zag and contiguous splits, and per owner the K and V base addresses,
the 4-D dims {64, Hkv, Tl, B}, the byte strides, the box and the swizzle,
plus the rejections (too many owners, a chunk that is not a whole number of
boxes, a misaligned base). Needs nvcc; no kernel is launched."""

import json
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

DRIVER = r'''
#include <cstdio>
#include <cstdlib>
#include "attention_peers.cuh"
using namespace g2b;

static int g_calls = 0;
static CUresult stub_encode(CUtensorMap* tm, CUtensorMapDataType dt, cuuint32_t rank, void* base,
                            const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                            const cuuint32_t* estr, CUtensorMapInterleave il, CUtensorMapSwizzle sw,
                            CUtensorMapL2promotion l2, CUtensorMapFloatOOBfill oob) {
  std::printf("{\"map\": %d, \"dtype\": %d, \"rank\": %u, \"base\": %llu, \"dims\": [%llu, %llu, %llu, %llu], "
              "\"strides\": [%llu, %llu, %llu], \"box\": [%u, %u, %u, %u], \"swizzle\": %d}\n",
              g_calls++, (int)dt, rank, (unsigned long long)(uintptr_t)base,
              (unsigned long long)dims[0], (unsigned long long)dims[1], (unsigned long long)dims[2],
              (unsigned long long)dims[3], (unsigned long long)strides[0], (unsigned long long)strides[1],
              (unsigned long long)strides[2], box[0], box[1], box[2], box[3],
              sw == CU_TENSOR_MAP_SWIZZLE_128B ? 128 : 0);
  return CUDA_SUCCESS;
}

int main(int argc, char** argv) {
  const int world = atoi(argv[1]), Tl = atoi(argv[2]), zigzag = atoi(argv[3]);
  const int Hkv = atoi(argv[4]), B = atoi(argv[5]), rows = atoi(argv[6]);
  const uintptr_t base0 = strtoull(argv[7], nullptr, 10);
  KvPeers p;
  p.world = world;
  p.zigzag = zigzag;
  p.Tl = Tl;
  for (int q = 0; q < world && q < kKvMaxOwners; ++q)
    p.base[q] = reinterpret_cast<void*>(base0 + (uintptr_t)q * (1u << 24));
  const int C = Hkv * 64;
  p.sb = (int64_t)Tl * 2 * C;
  p.st = 2 * C;
  p.v_off = C;
  static uint32_t flags[16];
  p.flags = flags;
  p.epoch = 7;
  KvPeerMaps m;
  const bool ok = make_kv_peer_maps(&m, p, Hkv, B, rows, &stub_encode);
  std::printf("{\"ok\": %d}\n", ok ? 1 : 0);
  if (!ok) return 0;
  std::printf("{\"owners\": [");
  for (int k = 0; k < world * Tl; ++k) {
    int lr = -1;
    const int q = kv_owner_row(m, k, &lr);
    std::printf("%s[%d, %d]", k ? ", " : "", q, lr);
  }
  std::printf("], \"epoch\": %u, \"world\": %d, \"flags_ok\": %d}\n", m.epoch, m.world,
              m.flags == flags ? 1 : 0);
  return 0;
}
'''


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    nvcc = shutil.which("nvcc") or ("/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc")
                                    else None)
    if nvcc is None:
        pytest.skip("nvcc not available")
    d = tmp_path_factory.mktemp("kvpeers")
    src = d / "drv.cu"
    src.write_text(DRIVER)
    exe = d / "drv"
    subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-I", os.path.join(ROOT, "csrc"),
                    str(src), "-o", str(exe)], check=True,
                   capture_output=True, timeout=600)
    return str(exe)


def _run(exe, world, Tl, zigzag, Hkv=2, B=3, rows=64, base0=1 << 32):
    out = subprocess.run([exe, str(world), str(Tl), str(zigzag), str(Hkv), str(B), str(rows), str(base0)],
                         check=True, capture_output=True, text=True, timeout=60).stdout
    recs = [json.loads(l) for l in out.splitlines() if l.strip()]
    maps = [r for r in recs if "map" in r]
    ok = [r for r in recs if "ok" in r][0]["ok"]
    owners = [r for r in recs if "owners" in r]
    return ok, maps, (owners[0] if owners else None)


def _expected_owner(k, world, Tl, zigzag):
    if not zigzag:
        return k // Tl, k % Tl
    h = Tl // 2
    c = k // h
    if c < world:
        return c, k % h
    return 2 * world - 1 - c, h + k % h


@pytest.mark.parametrize("world,Tl,zigzag", [(1, 128, 0), (2, 256, 0), (2, 256, 1), (4, 256, 1), (8, 256, 1),
                                             (8, 128, 0)])
def test_owner_rows_and_maps(driver, world, Tl, zigzag):
    Hkv, B, rows, base0 = 2, 3, 64, 1 << 32
    ok, maps, own = _run(driver, world, Tl, zigzag, Hkv, B, rows, base0)
    assert ok == 1
    C = Hkv * 64
    # one K map then one V map per owner, in owner order
    assert len(maps) == 2 * world
    for q in range(world):
        for which, m in enumerate(maps[2 * q: 2 * q + 2]):
            assert m["base"] == base0 + q * (1 << 24) + which * C * 2, (q, which, m)
            assert m["rank"] == 4 and m["swizzle"] == 128
            assert m["dims"] == [64, Hkv, Tl, B]
            assert m["strides"] == [128, 2 * C * 2, Tl * 2 * C * 2]
            assert m["box"] == [64, 1, rows, 1]
    assert own["epoch"] == 7 and own["world"] == world and own["flags_ok"] == 1
    got = [tuple(x) for x in own["owners"]]
    want = [_expected_owner(k, world, Tl, zigzag) for k in range(world * Tl)]
    assert got == want
    # every owner contributes exactly its Tl rows, each once
    for q in range(world):
        assert sorted(r for o, r in got if o == q) == list(range(Tl))


def test_rejections(driver):
    assert _run(driver, 9, 256, 1)[0] == 0                 # more owners than one NVSwitch domain
    assert _run(driver, 2, 192, 0, rows=128)[0] == 0       # Tl not a whole number of 128-row boxes
    assert _run(driver, 2, 128, 1, rows=128)[0] == 0       # zig-zag chunk of 64 rows under 128-row boxes
    assert _run(driver, 2, 256, 1, base0=(1 << 32) + 8)[0] == 0   # base not 16-byte aligned
    assert _run(driver, 2, 256, 1, rows=128)[0] == 1
