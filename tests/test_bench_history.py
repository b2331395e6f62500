"""Bench-history tooling (counterparts of the crate's examples/bench_quick.rs and
examples/bench_compare.rs): CSV format and the commit comparison, on CPU; the
timing run itself on a GPU."""
import pytest

from fa_b200 import bench_compare as bc
from fa_b200 import bench_quick as bq

ROW = "1700000000,{c},linux,x86_64,NVIDIA B200,{g},tf32,{v},{causal},1024,64,{t}"


def history(*rows):
    return "\n".join([bq.HEADER] + list(rows)) + "\n"


def test_csv_lines_match_the_schema():
    lines = bq.csv_lines([("v2", True, 1024, 64, 0.123456)], "abc1234", "NVIDIA B200", 1,
                         "tf32", 1700000000)
    assert lines[0] == bq.HEADER
    f = lines[1].split(",")
    assert len(f) == bc.N_FIELDS
    assert f[1] == "abc1234" and f[4] == "NVIDIA B200" and f[5] == "1" and f[6] == "tf32"
    assert f[7:11] == ["v2", "true", "1024", "64"] and f[11] == "0.1235"


def test_parse_skips_headers_and_malformed_rows():
    warnings = []
    text = history(ROW.format(c="a", g=1, v="v2", causal="true", t="1.0"),
                   "garbage,row",
                   bq.HEADER,  # a second concatenated run's header
                   ROW.format(c="b", g=1, v="v2", causal="maybe", t="1.0"),
                   ROW.format(c="b", g=1, v="v2", causal="true", t="0.9"))
    rows = bc.parse_csv(text, warn=warnings.append)
    assert [r.commit for r in rows] == ["a", "b"]
    assert len(warnings) == 2


def test_compare_joins_on_every_key_field():
    text = history(ROW.format(c="a", g=1, v="v2", causal="true", t="1.00"),
                   ROW.format(c="a", g=2, v="v2", causal="true", t="1.00"),
                   ROW.format(c="a", g=1, v="v1", causal="false", t="2.00"),
                   ROW.format(c="b", g=1, v="v2", causal="true", t="0.90"),
                   ROW.format(c="b", g=2, v="v2", causal="true", t="1.05"),
                   ROW.format(c="b", g=1, v="v3", causal="false", t="3.00"))
    rows = bc.parse_csv(text)
    assert bc.commits_in_order(rows) == ["a", "b"]
    res = {(k.gpus, k.variant): (o, n, m) for k, o, n, _, m in bc.compare(rows, "a", "b")}
    assert res[(1, "v2")][2] == "faster"      # -10 %
    assert res[(2, "v2")][2] == "SLOWER"      # +5 %
    assert res[(1, "v1")] == (2.0, None, "gone")
    assert res[(1, "v3")] == (None, 3.0, "new")


def test_compare_cli_resolves_prefixes(tmp_path, capsys):
    p = tmp_path / "history.csv"
    p.write_text(history(ROW.format(c="aaaa111", g=1, v="v2", causal="true", t="1.0"),
                         ROW.format(c="bbbb222", g=1, v="v2", causal="true", t="1.01")))
    assert bc.main(["--file", str(p), "aaaa", "bbbb"]) == 0
    out = capsys.readouterr().out
    assert "comparing aaaa111 -> bbbb222" in out and "~" in out
    with pytest.raises(SystemExit):
        bc.main(["--file", str(p), "cccc", "bbbb"])


def test_compare_cli_with_one_commit(tmp_path, capsys):
    p = tmp_path / "history.csv"
    p.write_text(history(ROW.format(c="aaaa111", g=1, v="v2", causal="true", t="1.0")))
    assert bc.main(["--file", str(p)]) == 0
    assert "nothing to compare yet" in capsys.readouterr().out


@pytest.mark.gpu
def test_bench_quick_measures_every_shape_and_variant(gpu_lib):
    rows = bq.measure(gpu_lib, iters_small=1, iters_large=1)
    keys = {(v, c, s, d) for v, c, s, d, _ in rows}
    for s, d in bq.SHAPES:
        for c in (False, True):
            for v in bq.VARIANTS + ("device",):
                assert (v, c, s, d) in keys
    assert all(t > 0 for *_, t in rows)
