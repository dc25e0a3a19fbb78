"""The benchmark's reference arm runs on the host cores, so its JSON contract
is checked here without a GPU: one line on stdout, the GPU arm's metric, unit,
direction and workload, a cpu_baseline of kind "reference" and an e2e entry
with no host/device bytes.  (When the compiled reference core is missing the
arm prints its "unavailable" line instead, which is checked too.)"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    sys.path.insert(0, ROOT)
    import bench
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    if "unavailable" in d:
        return
    assert d["metric"] == bench.METRIC and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["config"]["workload"] == bench.WORKLOAD
    assert d["value"] > 0 and d["steps"] >= 1
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_gpu_local_cpu_binding_with_a_fake_nvml(monkeypatch):
    """The e2e loop's pinned buffers are allocated on the CPUs NVML reports
    as local to the GPU: the affinity bit mask (64-bit words) is decoded,
    intersected with the allowed set, applied to the calling thread and
    undone afterwards; without NVML the thread is left alone."""
    import types
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    allowed = os.sched_getaffinity(0)
    want = sorted(allowed)[: max(1, len(allowed) // 2)]
    words = [0] * ((max(want) // 64) + 1)
    for c in want:
        words[c // 64] |= 1 << (c % 64)
    fake = types.SimpleNamespace(nvmlInit=lambda: None, nvmlDeviceGetHandleByIndex=lambda i: ("gpu", i),
                                 nvmlDeviceGetCpuAffinity=lambda h, n: words + [0] * max(0, n - len(words)))
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench._GpuLocalCpus(0) as b:
        assert os.sched_getaffinity(0) == set(want)
        assert b.note.startswith(f"{len(want)} GPU-local CPUs")
    assert os.sched_getaffinity(0) == allowed

    def broken():
        raise RuntimeError("no NVML")
    monkeypatch.setitem(sys.modules, "pynvml", types.SimpleNamespace(nvmlInit=broken))
    with bench._GpuLocalCpus(0) as b:
        assert os.sched_getaffinity(0) == allowed
        assert b.note.startswith("not bound")
