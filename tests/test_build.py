"""The build recipe's variant option (fuselse_b200.build): a build with shape
macros must name an output of its own, so it can never overwrite the in-tree
library that the tests and the bench load."""
import pytest

from fuselse_b200 import build as B


def test_defines_need_their_own_output():
    with pytest.raises(ValueError, match="output path of its own"):
        B.build(defines=["FL_FLAT_ROWS=0"])


def test_compile_command_carries_the_defines(tmp_path, monkeypatch):
    seen = {}

    class R:
        returncode, stdout, stderr = 0, "", ""

    def fake_run(cmd, capture_output, text):
        seen["cmd"] = cmd
        return R()

    monkeypatch.setattr(B.subprocess, "run", fake_run)
    src = B.CSRC / "vocab.cu"
    B._compile("nvcc", src, tmp_path / "vocab.o", False, False, ("FL_FLAT_ROWS=2",))
    assert "-DFL_FLAT_ROWS=2" in seen["cmd"]
    assert seen["cmd"][-2:] == ["-o", str(tmp_path / "vocab.o")]
