"""The repository's documents name only files that exist: every repo path in
backticks in DESIGN.md, INTEGRATION.md, README.md and profiles/README.md
(paths of the package, tests, oracle, profiles, the header, bench.py and
__graft_entry__.py; a csrc/ path is taken relative to the package)."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ROOTS = ("tensor-inference_b200/", "tests/", "oracle/", "profiles/", "include/ti_b200.h", "csrc/", "bench.py",
         "__graft_entry__.py")


@pytest.mark.parametrize("doc", ["DESIGN.md", "INTEGRATION.md", "README.md", "profiles/README.md"])
def test_documents_name_existing_files(doc):
    missing = []
    for tok in re.findall(r"`([^`\s]+)`", open(os.path.join(ROOT, doc)).read()):
        path = re.sub(r":\d[\d,\-]*$", "", tok.split("::")[0].rstrip(",.;:"))
        if not path.startswith(ROOTS) or any(c in path for c in "*{…<"):
            continue
        if not any(os.path.exists(os.path.join(ROOT, p)) for p in (path, os.path.join("tensor-inference_b200", path))):
            missing.append(tok)
    assert not missing, missing
