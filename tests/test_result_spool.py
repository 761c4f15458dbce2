"""Result spool (`utils/result_spool.py`): complete records reach the destination through the
independent copier, torn tails are not forwarded, and a writer killed mid-run loses nothing it had
flushed (CPU; the writer is this test's own child process, ended by its PID)."""
import json
import os
import subprocess
import sys
import time

from deepep_slingshot_b200.utils import result_spool as rs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_copy_pass_forwards_complete_lines_only(tmp_path):
    spool, dest = tmp_path / 'spool', tmp_path / 'dest'
    w = rs.SpoolWriter(str(spool), 'timings-rank0.jsonl')
    w.write({'i': 0})
    with open(spool / 'timings-rank0.jsonl', 'a') as f:
        f.write('{"i": 1')          # a torn record (writer died mid-line)
    offsets = {}
    rs.copy_pass(str(spool), str(dest), offsets)
    assert [json.loads(l) for l in open(dest / 'timings-rank0.jsonl')] == [{'i': 0}]
    with open(spool / 'timings-rank0.jsonl', 'a') as f:
        f.write('}\n')               # completed later: forwarded once, whole
    rs.copy_pass(str(spool), str(dest), offsets)
    assert [json.loads(l) for l in open(dest / 'timings-rank0.jsonl')] == [{'i': 0}, {'i': 1}]


WRITER = r'''
import sys, time
from deepep_slingshot_b200.utils import result_spool as rs
spool, dest = sys.argv[1], sys.argv[2]
rs.start_copier(spool, dest, interval=0.05)
w = rs.SpoolWriter(spool, 'correctness-rank0.jsonl')
for i in range(20):
    w.write({'case': i})
print('WRITTEN', flush=True)
time.sleep(600)   # hangs until killed
'''


def test_records_survive_a_killed_writer(tmp_path):
    spool, dest = str(tmp_path / 'spool'), str(tmp_path / 'dest')
    env = dict(os.environ, PYTHONPATH=ROOT)
    p = subprocess.Popen([sys.executable, '-c', WRITER, spool, dest], env=env, stdout=subprocess.PIPE, text=True)
    try:
        assert p.stdout.readline().strip() == 'WRITTEN'
    finally:
        p.kill()  # this test's own child, by PID
        p.wait()
    path = os.path.join(dest, 'correctness-rank0.jsonl')
    deadline = time.time() + 20
    got = []
    while time.time() < deadline:
        if os.path.exists(path):
            got = [json.loads(l) for l in open(path)]
            if len(got) == 20:
                break
        time.sleep(0.1)
    assert got == [{'case': i} for i in range(20)]


def test_done_marker_ends_the_copier(tmp_path):
    spool, dest = str(tmp_path / 'spool'), str(tmp_path / 'dest')
    os.makedirs(spool)
    t0 = time.time()
    w = rs.SpoolWriter(spool, 'manifest-rank0.jsonl')
    w.write({'m': 1})
    rs.finish(spool)
    rs.copy_loop(spool, dest, parent_pid=None, interval=0.05, max_seconds=10)
    assert time.time() - t0 < 5
    assert [json.loads(l) for l in open(os.path.join(dest, 'manifest-rank0.jsonl'))] == [{'m': 1}]
