"""The C-ABI library on the CPU: it loads, exports every entry point include/tabicl_b200.h declares, and its
host-only helpers agree with the oracle. No compute call needs a GPU here."""
import os
import re

import pytest

from conftest import ROOT, has_gpu, tcu
import oracle


def declared():
    text = open(os.path.join(ROOT, "include", "tabicl_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tcu_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_entry_point():
    names = declared()
    assert len(names) >= 25
    lib = tcu.lib()
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/tabicl_b200.h but not exported"


def test_record_sizes_agree_with_the_format():
    for kv in (0, 1, 2):
        for d, rc in [(512, 256), (16, 48), (32, 7), (512, 16)]:
            assert tcu.record(kv, d, rc) == oracle.record(kv, d, rc)


@pytest.mark.skipif(has_gpu(), reason="checks the no-device path")
def test_open_without_a_device_is_an_error_not_a_crash():
    with pytest.raises(tcu.TcuError):
        tcu.Gpu(0)


def test_bundle_round_trip(tmp_path):
    import numpy as np
    from tabicl_anywhere_b200 import tirs
    t = {"a": np.arange(6, dtype=np.float32).reshape(2, 3), "b": np.array([1, 2], np.int32),
         "c": np.frombuffer(b"xyz", np.uint8), "h": np.array([1.5, -2.0], np.float16)}
    p = tmp_path / "x.tirs"
    tirs.write(str(p), t)
    b = tirs.Bundle(str(p))
    assert b.names() == list(t)
    for k, v in t.items():
        assert np.array_equal(b[k], v)
    # every tensor on a 64-byte boundary (store.rs:7)
    assert all(off % 64 == 0 for (_, off, _, _) in b.entries.values())
