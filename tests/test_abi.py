"""CPU checks of the C-ABI boundary: the library loads without a GPU, exports every entry point that
include/sixi_smp.h and include/sixi_json.h declare, and the Python records match the C struct
layouts."""

from __future__ import annotations

import re
import subprocess
import textwrap

import pytest

from conftest import REPO

HEADER = REPO / "include" / "sixi_smp.h"
HEADERS = sorted((REPO / "include").glob("*.h"))
LIB = REPO / "sixi-asi_b200" / "lib" / "libsixi_smp.so"


def declared_symbols() -> list[str]:
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(sixi_(?:smp|json|schema)_[a-z_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    assert LIB.exists(), "build the library first (python sixi-asi_b200/build_lib.py)"
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (sixi_(?:smp|json|schema)_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    # nothing else leaks from the library (kernels and helpers are hidden)
    extra = sorted(s for s in exported if s not in declared_symbols())
    assert not extra, extra


def test_binding_declares_every_symbol():
    import sixi_smp

    assert sorted(sixi_smp.SIGNATURES) == declared_symbols()
    lib = sixi_smp.load()
    for name in declared_symbols():
        assert hasattr(lib, name)


def test_host_philox_matches_oracle_and_kat(port):
    import sixi_smp

    for seed, ctr, slot in [(0, 0, 0), (42, 7, 3), (2**63 + 5, 2**40 + 1, 8)]:
        assert sixi_smp.philox_uniform(seed, ctr, slot) == port.philox_uniform(seed, ctr, slot)


def test_status_strings_and_create_without_gpu():
    import ctypes

    import sixi_smp

    assert sixi_smp.status_string(0) == "Ok"
    assert sixi_smp.status_string(16) == "NumericNaNOrInf"
    h = ctypes.c_void_p()
    lib = sixi_smp.load()
    # invalid arguments are rejected before any device call
    assert lib.sixi_smp_create(0, 16, 0, ctypes.byref(h)) == sixi_smp.INVALID_ARGUMENT
    assert lib.sixi_smp_create(0, 16, 10_000_000, ctypes.byref(h)) == sixi_smp.INVALID_ARGUMENT
    assert lib.sixi_smp_sample(None, None, None, None, None, None, None, 0, None, None, None) == \
        sixi_smp.INVALID_ARGUMENT
    # NaN / Inf policy and suffix drafting: null handle, unknown policy, out-of-range sizes
    assert lib.sixi_smp_numeric_policy(None, None, 0, 0, 0, 0.0, None, None) == sixi_smp.INVALID_ARGUMENT
    assert lib.sixi_smp_suffix_draft(None, None, None, 1, 3, 16384, None, 8, None, None, None) == \
        sixi_smp.INVALID_ARGUMENT


def test_numeric_report_layout():
    """sixi_smp_numeric_report is 32 bytes with the fields where the binding and the oracle read them."""
    import numpy as np

    import sixi_smp
    from oracle import binding

    assert sixi_smp.NUMERIC_REPORT_DTYPE == binding.NUMERIC_REPORT
    r = np.zeros(2, sixi_smp.NUMERIC_REPORT_DTYPE)
    r["first_bad_index"] = [-1, 7]
    import torch

    assert sixi_smp.numeric_reports(torch.from_numpy(r.view(np.uint8).reshape(2, 32)))["first_bad_index"].tolist() == [-1, 7]


def test_struct_layouts(tmp_path):
    import sixi_smp

    src = tmp_path / "layout.c"
    src.write_text(textwrap.dedent(f"""
        #include <stddef.h>
        #include <stdio.h>
        #include "{HEADER}"
        int main(void) {{
            printf("%zu %zu %zu %zu %zu\\n", sizeof(sixi_smp_params), offsetof(sixi_smp_params, seed),
                   offsetof(sixi_smp_params, counter), sizeof(sixi_smp_rows), offsetof(sixi_smp_rows, row_stride));
            printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(sixi_smp_numeric_report),
                   offsetof(sixi_smp_numeric_report, emergency_clamped), offsetof(sixi_smp_numeric_report, status),
                   offsetof(sixi_smp_numeric_report, nan_count), offsetof(sixi_smp_numeric_report, inf_count),
                   offsetof(sixi_smp_numeric_report, first_bad_index));
            return 0;
        }}
    """))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", str(src), "-o", str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    pd = sixi_smp.PARAMS_DTYPE
    assert vals[0] == pd.itemsize
    assert vals[1] == pd.fields["seed"][1]
    assert vals[2] == pd.fields["counter"][1]
    assert vals[3] == __import__("ctypes").sizeof(sixi_smp.Rows)
    assert vals[4] == sixi_smp.Rows.row_stride.offset
    nd = sixi_smp.NUMERIC_REPORT_DTYPE
    assert vals[5:] == [nd.itemsize] + [nd.fields[f][1] for f in ("emergency_clamped", "status", "nan_count",
                                                                   "inf_count", "first_bad_index")]


@pytest.mark.parametrize("vocab", [1, 31, 5000, 151_936, 262_144])
def test_launch_plan_limits(vocab):
    """Vocabularies up to 262,144 are planned (checked through create's argument validation on a
    machine without a device: only the vocabulary check precedes the device query)."""
    import ctypes

    import sixi_smp

    h = ctypes.c_void_p()
    st = sixi_smp.load().sixi_smp_create(-1, 16, vocab, ctypes.byref(h))
    assert st == sixi_smp.INVALID_ARGUMENT  # device -1 is invalid, the vocabulary itself is accepted


def test_missing_library_fails_loudly(tmp_path):
    """No CPU fallback: with the CUDA library absent every entry of the binding raises."""
    import sys

    code = ("import sixi_smp as S\n"
            "for f in (lambda: S.Sampler(0, 1, 64), lambda: S.philox_uniform(1, 2, 0), lambda: S.status_string(0)):\n"
            "    try:\n"
            "        f()\n"
            "    except (ImportError, OSError):\n"
            "        continue\n"
            "    raise SystemExit('an entry point ran without the library')\n"
            "print('raised')\n")
    env = dict(__import__("os").environ, SIXI_SMP_LIB=str(tmp_path / "absent.so"))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120,
                       cwd=str(REPO / "sixi-asi_b200"))
    assert r.returncode == 0 and "raised" in r.stdout, (r.stdout, r.stderr[-1000:])


def test_verify_static_argument_checks_without_gpu():
    """sixi_smp_verify_static rejects bad arguments before any device call: device outside [0, 64),
    an empty vocabulary, k = 0, a row count that is not n_streams * (k + 1), null outputs and a
    misaligned draft_probs (SIXI_INVALID_ARGUMENT); more rows than its static workspace holds
    (SIXI_OUT_OF_BOUNDS)."""
    import ctypes

    import sixi_smp

    lib = sixi_smp.load()
    INV, OOB = sixi_smp.INVALID_ARGUMENT, sixi_smp.OUT_OF_BOUNDS
    V, k = 4097, 8
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: every call below returns before that
    outs = [fake] * 6

    def rows(n):
        return sixi_smp.Rows(fake.value, sixi_smp.F32, n, V)

    def call(device=0, vocab=V, n_rows=2 * (k + 1), n_streams=2, kk=k, q=None, outputs=None, target=True):
        r = rows(n_rows)
        return lib.sixi_smp_verify_static(device, vocab, ctypes.byref(r) if target else None, q, fake, None,
                                          n_streams, kk, fake, None, None, None, None, 0,
                                          *(outputs if outputs is not None else outs), None)

    assert call(device=-1) == INV
    assert call(device=64) == INV
    assert call(vocab=0) == INV
    assert call(kk=0, n_rows=2) == INV
    assert call(n_rows=2 * (k + 1) + 1) == INV
    assert call(target=False) == INV
    for i in range(6):
        o = list(outs)
        o[i] = None
        assert call(outputs=o) == INV, i
    limit = sixi_smp.STATIC_VERIFY_ROWS
    s = limit // (k + 1) + 1
    assert call(n_streams=s, n_rows=s * (k + 1)) == OOB
    assert call(q=ctypes.c_void_p(0x1002)) == INV
