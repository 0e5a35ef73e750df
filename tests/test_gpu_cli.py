"""The reference-compatible driver on the GPU: `branchcraft test` (the
reference's CPU-oracle gate), and the two benchmark modes with the reference's
CSV columns."""
import csv
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

CLI = Path(__file__).resolve().parent / "cli" / "branchcraft"


def test_branchcraft_test_mode():
    r = subprocess.run([str(CLI), "test"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "PASS 42 CPU-oracle checks" in r.stdout
    assert "PASS 3 tree CPU-oracle cases" in r.stdout


@pytest.mark.parametrize("mode,columns", [
    ("bench", "gpu,sm,cuda_runtime,batch,query_heads,kv_heads,head_dim,context,page_size,"
              "splits,single_us,split_us,speedup,max_abs_diff,kv_mib"),
    ("tree-bench", "gpu,sm,cuda_runtime,requests,tree_nodes,prefix_tokens,query_heads,kv_heads,"
                   "head_dim,page_size,tree_us,expanded_us,latency_ratio,max_abs_diff,"
                   "shared_kv_mib,expanded_kv_mib,memory_saving_pct"),
])
def test_bench_modes_quick(tmp_path, mode, columns):
    out = tmp_path / f"{mode}.csv"
    r = subprocess.run([str(CLI), mode, "--quick", "--output", str(out)], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    rows = list(csv.reader(out.open()))
    assert ",".join(rows[0]) == columns
    assert len(rows) == 5
