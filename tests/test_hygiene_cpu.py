"""Source hygiene: every logger of the package lives under ``vllm.b200``;
comments and docstrings state facts in their own words instead of pointing
at this project's planning notes; no source names the batched-copy CUDA
calls that are kept out of this code base."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
SOURCES = [p for pat in ("vllm_sm70_b200/**/*.py", "vllm_sm70_b200/**/*.cu",
                         "vllm_sm70_b200/**/*.cuh", "vllm_sm70_b200/**/*.h",
                         "vllm_sm70_b200/**/*.cpp", "*.py")
           for p in ROOT.glob(pat) if "_work" not in p.parts and "baseline" not in p.parts]
NOTES = re.compile(r"\b(SURVEY|DESIGN|VERDICT|ADVICE)\.md\b")
BATCHED = re.compile(r"cu(da)?Memcpy(3D)?Batch" + "Async")


def test_sources_found():
    assert len(SOURCES) > 50


def test_logger_names():
    bad = []
    for p in SOURCES:
        if p.suffix != ".py":
            continue
        for m in re.finditer(r"getLogger\(\s*[\"']([^\"']+)[\"']", p.read_text()):
            if not m.group(1).startswith("vllm.b200"):
                bad.append((str(p), m.group(1)))
    assert bad == []


def test_no_planning_note_references_or_closed_calls():
    bad = [str(p) for p in SOURCES if NOTES.search(p.read_text(errors="ignore"))
           or BATCHED.search(p.read_text(errors="ignore"))]
    assert bad == []


def test_native_env_knobs_registered():
    """Every VLLM_B200_* variable the native library reads is documented in
    the Python registry (envs.py), like the ones read from Python."""
    from vllm_sm70_b200 import envs

    names = set()
    for p in SOURCES:
        if p.suffix in (".cu", ".cuh", ".h", ".cpp"):
            names.update(re.findall(r'getenv\("(VLLM_B200_[A-Z0-9_]+)"\)', p.read_text()))
    assert names, "no native knobs found"
    missing = sorted(n for n in names if n not in envs._REGISTRY)
    assert missing == []
