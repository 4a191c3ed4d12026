"""bench.py's reference arm prints the JSON line a benchmark driver reads.

The arm times the oracle (the CPU restatement of gem's scoring path) on the host cores, so this runs
without a GPU: one bounded step of the 270M two-level workload in a child process, then checks the
base keys, a cpu_baseline describing the run, and an e2e with no host-device copies."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

BASE_KEYS = ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e")


def test_reference_arm_json_line():
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(ROOT / "prefix-head_b200"), str(ROOT)]))
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    run = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, run.stdout[-2000:]
    d = json.loads(lines[0])
    for k in BASE_KEYS:
        assert k in d, k
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0
    assert d["config"]["workload"] and "model" not in d["config"]
    pub = d["published_baseline"]  # the reference's own figure for this metric and workload
    assert pub["value"] == 308.6 and pub["unit"] == d["unit"]
    assert abs(d["vs_baseline"] - d["value"] / pub["value"]) < 0.01
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    gb = cb["gem_bench"]  # gem bench's JSONL fields (main.rs:295-310)
    assert gb["threads"] == cb["cores"] and gb["tokens"] == 512 and gb["body_us"] > 0 and gb["head_us"] > 0
    assert 0 < gb["head_share"] < 1 and abs(gb["tok_per_s"] - d["value"]) <= 0.02 * d["value"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_reference_arm_under_torchrun_prints_one_line():
    """Launched as the driver launches it for N > 1 (torchrun, one process per GPU), rank 0 alone times
    the CPU path and prints the line; the other rank exits 0 without work."""
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(ROOT / "prefix-head_b200"), str(ROOT)]))
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    run = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", "29531", str(ROOT / "bench.py"),
                          "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, run.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["cpu_baseline"]["value"] == d["value"]


def test_roofline_bytes_of_the_270m_geometry():
    """The roofline's denominators from the geometry alone (d 640, 18 layers, 4 q / 1 kv heads of 256,
    ff 2048, 2048 classes of 128): weights per step, and the algorithmic bytes of one scored token
    itemised in canonical GGUF sizes (Q8_0: 34 bytes per 32 weights; fp32 class table, bias and KV)."""
    import importlib
    sys.path.insert(0, str(ROOT))
    bench = importlib.import_module("bench")
    info = {"d": 640, "layers": 18, "head_dim": 256, "n_kv_heads": 1, "n_heads": 4, "ffn": 2048, "classes": 2048,
            "per": 128, "window": 512}
    weights = bench.body_weights(info)
    assert weights == 18 * (1024 * 640 + 2 * 256 * 640 + 640 * 1024 + 2 * 2048 * 640 + 640 * 2048) == 100_270_080
    info["body_bytes"] = weights // 32 * 34
    npos = bench.n_pos_schedule(info, 512)
    assert abs(npos.mean() - 256.5) < 1e-9  # every layer's window (512) covers the whole sequence
    body = 106_536_960
    classes = 2048 * 640 * 4 + 2048 * 4
    block = 128 * (640 + 20 * 2)            # one class block: 128 Q8_0 rows with f16 scales
    kv = 18 * 256.5 * 256 * 4 * 2 + 18 * 256 * 4 * 2
    vectors = 18 * (4 * 640 + 2 * 256 + 256) * 4 + 640 * 4
    want = body + classes + block + kv + vectors
    assert bench.bytes_per_token(info, npos, 0.0) == want == 121_609_728
    assert bench.bytes_per_token(info, npos, 1.0) == want + block  # the top class's block too


class _FakeNvml:
    """The NVML calls bench.Clocks makes, with a clock and reason bits that change between samples."""
    NVML_CLOCK_SM = 1

    def __init__(self):
        self.n = 0
        self.shut = False

    def nvmlInit(self):
        pass

    def nvmlShutdown(self):
        self.shut = True

    def nvmlDeviceGetHandleByUUID(self, uuid):
        raise RuntimeError("no CUDA device here")

    def nvmlDeviceGetHandleByIndex(self, i):
        return ("gpu", i)

    def nvmlDeviceGetMaxClockInfo(self, h, which):
        return 1965

    def nvmlDeviceGetClockInfo(self, h, which):
        self.n += 1
        return 1965 if self.n % 3 else 1800

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return 0x4 if self.n % 2 else 0x1  # sw_power_cap on odd samples; gpu_idle (not reported) on even


def test_clock_sampler_reads_nvml_during_the_region():
    """The sampler polls NVML from a thread while the region runs and reports the median SM clock, the
    maximum and the throttle reasons by nvidia-smi's field names; it only reads."""
    import importlib
    import time
    sys.path.insert(0, str(ROOT))
    bench = importlib.import_module("bench")
    fake = _FakeNvml()
    with bench.Clocks(0, nvml=fake) as clk:
        time.sleep(0.1)
    s = clk.summary()
    assert s["source"] == "nvml" and s["samples"] >= 5 and fake.shut
    assert s["sm_max_mhz"] == 1965 and s["sm_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]
    n = s["samples"]
    time.sleep(0.05)
    assert clk.summary()["samples"] == n  # nothing sampled after the region
