"""bench.py --impl reference on the host: the reference's CPU path (the oracle's
restatement of its CPU forward) runs the headline workload itself, prints the
repo arm's `config`, and loads nothing of the library it is compared with."""
import json
import subprocess
import sys

from conftest import ROOT

CODE = """
import json, sys
sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '0']
import bench
bench.main()
maps = open('/proc/self/maps').read()
assert 'liblsx.so' not in maps, 'the library was loaded'
assert 'laplacesscissors_b200' not in sys.modules, 'the package was imported'
print(json.dumps({'config': bench.decode_config(1)}))
"""


def test_reference_arm_runs_the_workload_without_the_library():
    r = subprocess.run([sys.executable, "-c", CODE], cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(x) for x in r.stdout.strip().splitlines() if x.startswith("{")]
    line, expected = lines[-2], lines[-1]["config"]
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["value"] > 0
    assert line["config"] == expected
    assert line["config"]["decode_steps_per_step"] == 55
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert len(line["first_tokens"]) == 8
