"""The C-ABI library loads without a GPU and exports every symbol its header
declares; the Python drop-in keeps the reference's entry names and rejects bad
arguments before touching a device."""
import ctypes
import os
import re

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "hyperion_b200.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(hyperion_[a-z_]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_expected_entry_points():
    names = _declared_functions()
    assert "hyperion_apex_kernel" in names and "hyperion_reset_counter" in names
    from hyperion_b200 import _capi

    assert set(names) == set(_capi.EXPORTED)


def test_library_loads_and_exports_every_declared_symbol(hyperion):
    lib = ctypes.CDLL(hyperion.library_path())
    for name in _declared_functions():
        assert hasattr(lib, name), name
    assert lib.hyperion_version() == 10400


def test_drop_in_names_match_reference_module(hyperion):
    # hyperion_fa3_production_final.py:598-601 binds exactly these two names.
    assert callable(hyperion.hyperion_apex_kernel)
    assert callable(hyperion.hyperion_reset_counter)
    assert hyperion.HYPERION_LOADED is True


def test_python_boundary_rejects_cpu_tensors(hyperion):
    t = torch.zeros(4, 4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        hyperion.hyperion_apex_kernel(t, 4, t, None, t, None, t.to(torch.uint8), torch.ones(1), t[0],
                                      None, torch.zeros(4, 128), 1, 128, 16, 16, 1, 0.088, False)


def test_c_boundary_rejects_bad_sizes_without_touching_the_device(hyperion):
    from hyperion_b200 import _capi

    lib = _capi.lib
    ext = _capi.Extents(1, 16, 1, 0, _capi.DTYPE_F32, 0, 0, 0)
    fake = ctypes.c_void_p(256)
    args = [fake, 1, fake, None, fake, None, fake, fake, fake, None, fake, 1, 128, 64, 16, 1,
            ctypes.c_float(0.088), 0, ctypes.byref(ext), fake, 1 << 20, None]
    # k_packed_bytes 64 is the reference's INT4 value; sign-bit K needs head_dim/8.
    assert lib.hyperion_apex_kernel(*args) == _capi.HYPERION_ERR_INVALID_ARG
    assert "k_packed_bytes" in _capi.last_error()
    args[13] = 16
    args[12] = 96
    assert lib.hyperion_apex_kernel(*args) == _capi.HYPERION_ERR_UNSUPPORTED
    args[12] = 128
    args[11] = 0  # seq_q
    assert lib.hyperion_apex_kernel(*args) == _capi.HYPERION_ERR_INVALID_ARG
    args[11] = 1
    args[19] = None  # workspace
    assert lib.hyperion_apex_kernel(*args) == _capi.HYPERION_ERR_WORKSPACE
    ext_bad = _capi.Extents(1, 16, 1, 5, _capi.DTYPE_F32, 0, 0, 0)  # table numel without pointer
    args[19] = fake
    args[18] = ctypes.byref(ext_bad)
    assert lib.hyperion_apex_kernel(*args) == _capi.HYPERION_ERR_INVALID_ARG


def test_c_boundary_rejects_bad_kv_group_without_touching_the_device(hyperion):
    from hyperion_b200 import _capi

    lib = _capi.lib
    ext = _capi.Extents(1, 16, 1, 0, _capi.DTYPE_F32, 0, 0, 0)
    fake = ctypes.c_void_p(256)

    def call(opt, ext_):
        return lib.hyperion_apex_kernel_ex(fake, 1, fake, None, fake, None, fake, fake, fake, None, fake, 1, 128, 16,
                                           16, 1, ctypes.c_float(0.088), 0, ctypes.byref(ext_), ctypes.byref(opt),
                                           fake, 1 << 20, None)

    assert call(_capi.Options(0, 0, None, 0, -1), ext) == _capi.HYPERION_ERR_INVALID_ARG
    assert "kv_group" in _capi.last_error()
    big = _capi.Extents(1 << 28, 16, 1, 0, _capi.DTYPE_F32, 0, 0, 0)
    assert call(_capi.Options(0, 0, None, 0, 16), big) == _capi.HYPERION_ERR_INVALID_ARG
    assert "kv_group" in _capi.last_error()


def test_python_boundary_checks_kv_group(hyperion):
    t = torch.zeros(4, 4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="kv_group"):
        hyperion.hyperion_apex_kernel(t, 4, t, None, t, None, t.to(torch.uint8), torch.ones(1), t[0],
                                      None, torch.zeros(4, 128), 1, 128, 16, 16, 1, 0.088, False, kv_group=0)


def test_ctypes_structs_match_the_c_header_layout(tmp_path):
    """The ctypes mirrors of hyperion_extents and hyperion_options must have the C
    header's field offsets and sizes; a C program compiled against the header
    prints them."""
    import shutil
    import subprocess

    from hyperion_b200 import _capi

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    structs = {"hyperion_extents": _capi.Extents, "hyperion_options": _capi.Options}
    lines = ['#include "hyperion_b200.h"', "#include <stdio.h>", "#include <stddef.h>", "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "abi.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "abi"
    subprocess.run([gcc, "-std=c99", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {tuple(line.split()[:2]): int(line.split()[2]) for line in out if line.strip()}
    for cname, cls in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, (cname, fname)


def test_c_boundary_accepts_an_empty_call_from_an_idle_rank(hyperion):
    """A rank that owns no (batch, head) row (more ranks than KV heads) calls with
    total_work 0 and empty tensors: nothing to launch, status OK, device untouched."""
    from hyperion_b200 import _capi

    ext = _capi.Extents(0, 0, 0, 0, _capi.DTYPE_BF16, 0, 0, 0)
    rc = _capi.lib.hyperion_apex_kernel(None, 0, None, None, None, None, None, None, None, None, None, 1, 128, 16,
                                        16, 1, ctypes.c_float(0.088), 1, ctypes.byref(ext), None, 0, None)
    assert rc == _capi.HYPERION_OK
    out = (ctypes.c_int32 * 4)()
    _capi.lib.hyperion_last_call_info(out, 4)
    assert list(out) == [0, 0, 0, 0]
    # Scalar arguments are still checked.
    rc = _capi.lib.hyperion_apex_kernel(None, 0, None, None, None, None, None, None, None, None, None, 1, 96, 12,
                                        16, 1, ctypes.c_float(0.088), 1, ctypes.byref(ext), None, 0, None)
    assert rc == _capi.HYPERION_ERR_UNSUPPORTED


def test_launch_table_is_a_measured_grid():
    """csrc/launch_table.h (written by tune_launch.py from a sweep on B200) holds one
    entry per measured shape: split counts among the swept candidates, and for each
    entry the time of its split no worse than the rule's at the same shape."""
    import os
    import re

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "hyperion-fa3-kernel-_b200",
                        "csrc", "launch_table.h")
    text = open(path).read()
    assert "kSplitTableSms = 148" in text
    rows = re.findall(r"\{(\d), (\d+), (\d+), (\d+)\},\s+// ([\d.]+) ms; the rule's (\d+): ([\d.]+) ms", text)
    assert len(rows) >= 30
    seen = set()
    for kernel, items, keys, splits, best_ms, rule, rule_ms in rows:
        assert (kernel, items, keys) not in seen
        seen.add((kernel, items, keys))
        assert int(splits) in (1, 2, 3, 4, 6, 8, 12, 16)
        assert float(best_ms) <= float(rule_ms) * 1.01
    assert {k for k, _, _ in seen} == {"0", "1", "2"}
