"""Host-side checks of bench.py's cost model and launch bookkeeping (CPU)."""
import json

import numpy as np

import bench


def test_layer_costs_sum_to_the_step_contraction():
    """The 25 GEMMs plus the stage-5 tail's three 32x32 projections account for
    the 706.7 MFLOP of dense contraction per latent frame (the tail's final
    32 -> 1 conv runs on CUDA cores and is not counted)."""
    for precision in (0, 1):
        costs = bench.layer_costs(precision)
        assert len(costs) == len(bench.kernel_names(precision)) == (17 if precision == 0 else 21)
        assert sum(c["flops"] for c in costs) == bench.FLOPS_PER_FRAME


def test_launch_order_is_one_default_step():
    # stem; stages 0-1: conv + 3 x (depthwise pre-pass, GEMM); stages 2-4: conv + fused stage;
    # stage 5: conv + tail
    assert len(bench.LAUNCH_ORDER) == 1 + 2 * 7 + 3 * 2 + 2 == 23
    assert set(bench.LAUNCH_ORDER) == set(bench.kernel_names(0))


def test_kernel_ms_folds_fused_layers():
    v = np.arange(26, dtype=np.float64)
    k = bench.kernel_ms(v, 0)
    names = bench.kernel_names(0)
    assert len(k) == len(names) and abs(k.sum() - v.sum()) < 1e-9
    assert k[names.index("stage3.units")] == 14 + 15 + 16
    assert k[names.index("stage5.tail")] == 22 + 23 + 24 + 25
    k8 = bench.kernel_ms(v, 1)
    names8 = bench.kernel_names(1)
    assert k8[names8.index("stage3.res1")] == 15 and k8[names8.index("stage4.units")] == 18 + 19 + 20


def test_tensor_roofline_fraction():
    pk = {"tflops": 1000.0, "source": "test"}
    r = bench.tensor_roofline(frames=1000, dev_s=0.001, e2e_s=0.002, pk=pk)
    assert abs(r["device_tflops"] - 706.740) < 0.01
    assert abs(r["device_frac"] - 0.7067) < 1e-4 and abs(r["e2e_frac"] - 0.3534) < 1e-4


def test_roofline_names_the_binding_pipe():
    pk = {"hbm_gbs": 6000.0, "tflops": 1400.0, "sm_mhz": 1965.0, "source": "test"}
    layer_ms = [0.1] * 16 + [0.5]  # the tail dominates
    r = bench.roofline(layer_ms, 512, 512, pk, "stream40ms", 1, 0)
    assert r["kernel"] == "stage5.tail" and r["bound"] in ("hbm", "tensor")
    assert r["binding"] == "cuda_core"
    assert 0 < r["cuda_core"]["frac"] < 1
    json.dumps(r)


def test_ingest_ncu_maps_launches_to_layers(tmp_path, monkeypatch):
    rows = ['"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"']
    for i, name in enumerate(bench.LAUNCH_ORDER):
        rows.append(f'"{i}","k{name}","dram__bytes_read.sum","Mbyte","1.5"')
        rows.append(f'"{i}","k{name}","dram__bytes_write.sum","byte","10"')
        rows.append(f'"{i}","k{name}","gpu__time_duration.sum","usecond","3"')
    csv_path = tmp_path / "launches.csv"
    csv_path.write_text("==PROF== noise\n" + "\n".join(rows) + "\n")
    out = tmp_path / "traffic.json"
    monkeypatch.setattr(bench, "TRAFFIC_FILE", out)
    bench.ingest_ncu(str(csv_path))
    d = json.loads(out.read_text())
    assert d["layers"]["stage5.tail"] == 1_500_010
    assert d["layers"]["stage0.res0"] == 2 * 1_500_010  # depthwise pre-pass + GEMM
