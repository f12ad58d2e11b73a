"""Host-side guarantees of the product package that need no GPU: it has no CPU
path and never reaches the oracle."""

import ast
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PACKAGE = ROOT / "sheetsage2_refined_b200"


def test_package_never_imports_the_oracle():
    for path in sorted(PACKAGE.rglob("*.py")):
        tree = ast.parse(path.read_text(), filename=str(path))
        for node in ast.walk(tree):
            if isinstance(node, ast.Import):
                names = [a.name for a in node.names]
            elif isinstance(node, ast.ImportFrom):
                names = [node.module or ""]
            else:
                continue
            assert not any(n == "oracle" or n.startswith("oracle.") for n in names), f"{path} imports {names}"
    for path in sorted((PACKAGE / "csrc").iterdir()):
        assert "oracle" not in path.read_text(errors="ignore"), f"{path} names the oracle"


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU refusal")
def test_batch_decoder_refuses_to_run_without_cuda():
    from sheetsage2_refined_b200 import BatchDecoder

    with pytest.raises(RuntimeError, match="no CPU path"):
        BatchDecoder(object(), object(), batch=1, frames=16)


def test_load_sources_are_held_until_their_copies_complete(monkeypatch):
    """``BatchDecoder._retain`` keeps each load's sources until the event recorded after its copies has completed."""

    import types

    from sheetsage2_refined_b200 import BatchDecoder

    class FakeEvent:
        done = set()
        count = 0

        def __init__(self):
            FakeEvent.count += 1
            self.id = FakeEvent.count

        def record(self, stream):
            self.stream = stream

        def query(self):
            return self.id in FakeEvent.done

    monkeypatch.setattr(torch.cuda, "Event", FakeEvent)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: "stream")
    eng = types.SimpleNamespace(_inflight=[], device=torch.device("cpu"))
    for i in range(3):
        BatchDecoder._retain(eng, (f"memory{i}", None))
    assert [s[0] for _, s in eng._inflight] == ["memory0", "memory1", "memory2"]
    FakeEvent.done.update({1, 2})  # the first two loads' copies have run
    BatchDecoder._retain(eng, ("memory3", None))
    assert [s[0] for _, s in eng._inflight] == ["memory2", "memory3"]
