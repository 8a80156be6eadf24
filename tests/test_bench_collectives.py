"""bench.py's multi-rank plumbing: every rank takes the same collective
steps.  A collective that only rank 0 reaches waits for ever (until the
process group's timeout), so none may sit inside an `if d.rank == 0` block;
and the Dist helper's reductions work across two gloo ranks on the CPU."""
import ast
import os
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COLLECTIVES = {"allsum", "allmax", "gather", "barrier"}


def _rank_guarded(node):
    t = node.test
    return (isinstance(t, ast.Compare) and isinstance(t.left, ast.Attribute) and t.left.attr == "rank"
            and len(t.ops) == 1 and isinstance(t.ops[0], ast.Eq))


def test_no_collective_inside_a_rank_zero_block():
    tree = ast.parse(open(os.path.join(ROOT, "bench.py")).read())
    bad = []
    for node in ast.walk(tree):
        if isinstance(node, ast.If) and _rank_guarded(node):
            for inner in node.body:
                for sub in ast.walk(inner):
                    if isinstance(sub, ast.Call) and isinstance(sub.func, ast.Attribute) \
                            and sub.func.attr in COLLECTIVES:
                        bad.append(sub.lineno)
    assert not bad, f"collectives inside rank-0 blocks at bench.py lines {bad}"


def test_dist_helpers_over_two_gloo_ranks(tmp_path):
    script = tmp_path / "ranks.py"
    script.write_text(textwrap.dedent(f"""
        import os, sys
        sys.path.insert(0, {ROOT!r})
        import bench
        d = bench.Dist()
        assert d.world == 2
        assert d.allsum(d.rank + 1) == 3.0
        assert d.allmax(10.0 * d.rank) == 10.0
        assert d.gather([d.rank]) == [[0], [1]]
        d.barrier()
        d.close()
        open(os.path.join({str(tmp_path)!r}, "ok%d" % d.rank), "w").close()
    """))
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                          "--master-addr", "127.0.0.1", "--master-port", "29533", str(script)],
                         env=env, capture_output=True, text=True, timeout=240)
    assert out.returncode == 0, out.stderr[-2000:]
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()
