"""The product package stays separate from the test infrastructure: no module under
qwen3_tts_b200/ imports the CPU oracle or the tests, and importing the package loads
neither (the GPU path has no CPU fallback to route through)."""
import ast
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PACKAGE = ROOT / "qwen3-tts-rsi-engine_b200" / "qwen3_tts_b200"


def imported_roots(path: Path) -> set:
    roots = set()
    for node in ast.walk(ast.parse(path.read_text())):
        if isinstance(node, ast.Import):
            roots.update(alias.name.split(".")[0] for alias in node.names)
        elif isinstance(node, ast.ImportFrom) and node.level == 0 and node.module:
            roots.add(node.module.split(".")[0])
    return roots


def test_no_product_module_imports_the_oracle_or_the_tests():
    offenders = {p.name: sorted(imported_roots(p) & {"oracle", "tests"}) for p in PACKAGE.glob("*.py")}
    assert not {k: v for k, v in offenders.items() if v}


def test_importing_every_product_module_loads_no_oracle(tmp_path):
    names = sorted(p.stem for p in PACKAGE.glob("*.py") if p.stem != "__init__")
    code = ("import sys\n"
            f"sys.path.insert(0, {str(PACKAGE.parent)!r})\n"
            f"for name in {names!r}:\n"
            "    __import__('qwen3_tts_b200.' + name)\n"
            "print(sorted(m for m in sys.modules if m.split('.')[0] in ('oracle', 'tests')))\n")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                         cwd=tmp_path)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == "[]"
