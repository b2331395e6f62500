"""Compares two commits' rows of a bench history CSV (``fa_b200.bench_quick --csv``).

The counterpart of the crate's ``examples/bench_compare.rs``: rows are joined
on every column except ``timestamp`` and ``time_ms`` (os, arch, device, gpus,
precision, variant, causal, seq_len, d_head), so different devices, GPU counts
or precisions are never compared by accident; a change of 3 % or more is
marked ``faster`` / ``SLOWER``.

    python -m fa_b200.bench_compare                 # last two distinct commits
    python -m fa_b200.bench_compare <old> <new>     # specific commits (prefix match)
    python -m fa_b200.bench_compare --file PATH ... # another history file

The default file is ``benches/history.csv`` next to the package.
"""
from __future__ import annotations

import os
import sys
from typing import NamedTuple

KEY_FIELDS = ("os", "arch", "device", "gpus", "precision", "variant", "causal", "seq_len",
              "d_head")
N_FIELDS = 12


class Key(NamedTuple):
    os: str
    arch: str
    device: str
    gpus: int
    precision: str
    variant: str
    causal: bool
    seq_len: int
    d_head: int


class Row(NamedTuple):
    commit: str
    key: Key
    time_ms: float


def default_path() -> str:
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    return os.path.join(here, "benches", "history.csv")


def parse_csv(text: str, warn=None):
    """Rows of the history; header lines (one per concatenated run) and
    malformed lines are skipped (reported through ``warn``)."""
    rows = []
    for line in text.splitlines():
        if not line or line.startswith("timestamp,"):
            continue
        f = line.split(",")
        if len(f) != N_FIELDS:
            if warn:
                warn(f"skipping malformed row: {line}")
            continue
        try:
            key = Key(f[2], f[3], f[4], int(f[5]), f[6], f[7],
                      {"true": True, "false": False}[f[8]], int(f[9]), int(f[10]))
            t = float(f[11])
        except (ValueError, KeyError):
            if warn:
                warn(f"skipping malformed row: {line}")
            continue
        rows.append(Row(f[1], key, t))
    return rows


def commits_in_order(rows):
    """Distinct commits in order of first appearance (history is append-only)."""
    out = []
    for r in rows:
        if r.commit not in out:
            out.append(r.commit)
    return out


def resolve(commits, arg: str) -> str:
    for c in commits:
        if c == arg or c.startswith(arg):
            return c
    raise SystemExit(f"no data for commit matching {arg!r}; known commits: {commits}")


def compare(rows, old: str, new: str):
    """(key, old_ms or None, new_ms or None, pct or None, marker) for every key."""
    om = {r.key: r.time_ms for r in rows if r.commit == old}
    nm = {r.key: r.time_ms for r in rows if r.commit == new}
    out = []
    for key in sorted(set(om) | set(nm)):
        o, n = om.get(key), nm.get(key)
        if o is not None and n is not None:
            pct = (n - o) / o * 100.0
            marker = "faster" if pct <= -3.0 else ("SLOWER" if pct >= 3.0 else "~")
            out.append((key, o, n, pct, marker))
        elif n is not None:
            out.append((key, None, n, None, "new"))
        else:
            out.append((key, o, None, None, "gone"))
    return out


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    path = default_path()
    if "--file" in argv:
        i = argv.index("--file")
        path = argv[i + 1]
        del argv[i:i + 2]
    with open(path) as fh:
        rows = parse_csv(fh.read(), warn=lambda m: print(m, file=sys.stderr))
    if not rows:
        print(f"no usable rows in {path}", file=sys.stderr)
        return 1
    commits = commits_in_order(rows)
    if len(argv) == 2:
        old, new = resolve(commits, argv[0]), resolve(commits, argv[1])
    elif len(commits) >= 2:
        old, new = commits[-2], commits[-1]
    else:
        print(f"only one commit ({commits[0]}) in {path} so far - nothing to compare yet. "
              "Append another `python -m fa_b200.bench_quick --csv` run after a change.")
        return 0
    print(f"comparing {old} -> {new}\n")
    print(f"{'device':<22} {'gpus':>4} {'prec':>6} {'var':>6} {'causal':>6} {'seq':>5} "
          f"{'d':>4} | {'old_ms':>10} {'new_ms':>10} {'change':>8}")
    only_old = only_new = 0
    for key, o, n, pct, marker in compare(rows, old, new):
        head = (f"{key.device[:22]:<22} {key.gpus:>4} {key.precision:>6} {key.variant:>6} "
                f"{str(key.causal).lower():>6} {key.seq_len:>5} {key.d_head:>4} | ")
        if marker == "gone":
            only_old += 1
        elif marker == "new":
            only_new += 1
            print(head + f"{'-':>10} {n:>10.4f} {'new':>9}")
        else:
            print(head + f"{o:>10.4f} {n:>10.4f} {pct:>+7.1f}% {marker}")
    if only_old:
        print(f"\n{only_old} measurement(s) present only in {old}, not in {new} "
              "(target/shape not re-measured)")
    if only_new:
        print(f"{only_new} measurement(s) present only in {new}, not in {old} "
              "(new target/shape, printed above as \"new\")")
    return 0


if __name__ == "__main__":
    import signal
    signal.signal(signal.SIGPIPE, signal.SIG_DFL)  # quiet when piped into head
    sys.exit(main())
