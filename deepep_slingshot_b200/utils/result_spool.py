"""Result spool: benchmark journals written to local memory-backed storage and copied out by an
independent process, so records that were written survive a benchmark process that hangs or dies.

The reference writes its JSONL journals through tmpfs with a separate copier process
(backend/tests/result_spool.py:23-104), because its output file system could stall or lose a
writer's tail when a job was killed. Here:
  * `SpoolWriter(name)` appends JSON lines to `<spool dir>/<name>` (default `/dev/shm/deepep_b200_spool/
    <job>`), flushing each record;
  * `start_copier(spool, dest)` launches `python -m deepep_slingshot_b200.utils.result_spool --copy
    <spool> <dest>` as its own process (a new session, so a signal to the benchmark's process group
    does not reach it). It appends every complete new line of every journal to the same name under
    `dest`, keeps an offset per file, and exits once `finish(spool)` wrote the done marker and
    everything is copied, or when its parent process is gone and a last pass is done;
  * only complete lines are copied: a record torn by a killed writer is never forwarded.
"""
import argparse
import json
import os
import subprocess
import sys
import time
from typing import Dict, Optional

DONE = '.done'


def default_spool_dir(job: str) -> str:
    base = '/dev/shm' if os.path.isdir('/dev/shm') else '/tmp'
    return os.path.join(base, 'deepep_b200_spool', job)


class SpoolWriter:
    """Append-only JSONL journal in the spool directory (one record per line, flushed)."""

    def __init__(self, spool_dir: str, name: str) -> None:
        os.makedirs(spool_dir, exist_ok=True)
        self.f = open(os.path.join(spool_dir, name), 'a')

    def write(self, rec: dict) -> None:
        self.f.write(json.dumps(rec) + '\n')
        self.f.flush()

    def close(self) -> None:
        self.f.close()


def finish(spool_dir: str) -> None:
    """Tell the copier that no more records will come (it exits after its last pass)."""
    with open(os.path.join(spool_dir, DONE), 'w') as f:
        f.write(str(time.time()))


def copy_pass(spool_dir: str, dest_dir: str, offsets: Dict[str, int]) -> int:
    """Append the complete new lines of every journal to `dest_dir`; returns the bytes copied."""
    moved = 0
    os.makedirs(dest_dir, exist_ok=True)
    for name in sorted(os.listdir(spool_dir)):
        if name == DONE:
            continue
        src = os.path.join(spool_dir, name)
        if not os.path.isfile(src):
            continue
        with open(src, 'rb') as f:
            f.seek(offsets.get(name, 0))
            data = f.read()
        end = data.rfind(b'\n')
        if end < 0:
            continue
        chunk = data[:end + 1]
        with open(os.path.join(dest_dir, name), 'ab') as out:
            out.write(chunk)
            out.flush()
            os.fsync(out.fileno())
        offsets[name] = offsets.get(name, 0) + len(chunk)
        moved += len(chunk)
    return moved


def _alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    return True


def copy_loop(spool_dir: str, dest_dir: str, parent_pid: Optional[int], interval: float = 0.2,
              max_seconds: float = 86400.0) -> None:
    """Copy until the done marker exists (or the parent is gone), then make a last pass."""
    offsets: Dict[str, int] = {}
    start = time.time()
    while time.time() - start < max_seconds:
        done = os.path.exists(os.path.join(spool_dir, DONE))
        orphan = parent_pid is not None and not _alive(parent_pid)
        copy_pass(spool_dir, dest_dir, offsets)
        if done or orphan:
            copy_pass(spool_dir, dest_dir, offsets)
            return
        time.sleep(interval)


def start_copier(spool_dir: str, dest_dir: str, interval: float = 0.2) -> subprocess.Popen:
    """The copier as an independent process (own session) watching this process."""
    os.makedirs(spool_dir, exist_ok=True)
    cmd = [sys.executable, '-m', 'deepep_slingshot_b200.utils.result_spool', '--copy', spool_dir, dest_dir,
           '--parent', str(os.getpid()), '--interval', str(interval)]
    return subprocess.Popen(cmd, start_new_session=True, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument('--copy', nargs=2, metavar=('SPOOL', 'DEST'), required=True)
    p.add_argument('--parent', type=int, default=None)
    p.add_argument('--interval', type=float, default=0.2)
    args = p.parse_args(argv)
    copy_loop(args.copy[0], args.copy[1], args.parent, args.interval)


if __name__ == '__main__':
    main()
