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
