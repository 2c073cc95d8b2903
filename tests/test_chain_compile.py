"""Run-time chain compilation on the host (NVRTC compiles to an sm_100a cubin
without a GPU): every op and operand form the golden chains use compiles, the
mode switch works, bad chains are refused before any compilation, and a chain
structure compiles once whatever its constant values."""
import numpy as np
import pytest

import mlk2_b200 as mb
from mlk2_b200 import api, kir

A, B, C, S, T, E = kir.A, kir.B, kir.C, kir.S, kir.T, kir.E


def _nvrtc_or_skip():
    prev = api.chain_compile(-1)[0]
    api.chain_compile(1)
    active = api.chain_compile(-1)[0]
    if not prev:
        api.chain_compile(0)
    if not active:
        pytest.skip("NVRTC is not loadable on this host")


@pytest.mark.parametrize("dtype", ["f32", "f64"])
@pytest.mark.parametrize("poly7", [False, True])
def test_every_golden_chain_compiles(golden, dtype, poly7):
    _nvrtc_or_skip()
    g = golden("chains")
    for name in [k[2:] for k in g.files if k.startswith("c_")]:
        ch = g["c_" + name]
        uses_b = any(int(e["a_kind"]) == 2 or int(e["b_kind"]) == 2 for e in ch)
        api.chain_build(ch, dtype=dtype, has_b=uses_b, poly7=poly7)


def test_every_op_in_one_chain_compiles():
    _nvrtc_or_skip()
    unary = ("neg", "exp", "log", "sin", "cos", "tan", "tanh", "sqrt", "rsqrt", "erf", "gelu")
    ex = [E("mul", A, C(0.125))]
    for op in ("add", "sub", "mul", "div", "pow") + unary:
        ex.append(E(op, T(len(ex) - 1)) if op in unary else E(op, T(len(ex) - 1), B))
    api.chain_build(kir.chain(*ex), dtype="f32", has_b=True)
    # the longest chain the ABI admits (64 expressions)
    long = [E("mul", A, C(1.0))] + [E("add", T(k), C(k)) for k in range(63)]
    api.chain_build(kir.chain(*long), dtype="f64")


def test_structure_compiles_once_whatever_the_constants():
    _nvrtc_or_skip()
    _, before, _ = api.chain_compile(-1)
    for v in (1.0, 2.0, -3.5, 1e300):
        api.chain_build(kir.chain(E("mul", A, C(v)), E("sub", T(0), S(3)), E("exp", T(1))),
                        dtype="f32")
    _, after, _ = api.chain_compile(-1)
    assert after - before <= 1


def test_mode_switch():
    _nvrtc_or_skip()
    try:
        assert api.chain_compile(0)[0] is False
        assert api.chain_compile(-1)[0] is False       # a query changes nothing
        assert api.chain_compile(7)[0] is False        # neither does an unknown mode
        assert api.chain_compile(1)[0] is True
    finally:
        api.chain_compile(1)


def test_bad_chains_refused_before_compiling():
    _, before, _ = api.chain_compile(-1)
    bad_op = kir.chain(E("mul", A, A))
    bad_op["op"][0] = 99
    with pytest.raises(mb.MLKBError):
        api.chain_build(bad_op)
    forward_temp = kir.chain(E("add", T(1), A), E("mul", A, A))
    with pytest.raises(mb.MLKBError):
        api.chain_build(forward_temp)
    with pytest.raises(mb.MLKBError):                  # ElemB without a b buffer
        api.chain_build(kir.chain(E("mul", A, B)), has_b=False)
    _, after, _ = api.chain_compile(-1)
    assert after == before


def _plan(chains, **kw):
    m = api.Module(kir.map_module(chains, **kw))
    return m.plan([mb.F64 if kw.get("dtype") == "f64" else mb.F32] * m.num_buffers)


def test_roots_over_the_same_inputs_share_one_kernel():
    two_x = kir.chain(E("mul", A, C(2.0)))
    cube = kir.chain(E("mul", A, A), E("mul", T(0), A))
    # no dedicated kernel applies (poly7 family): one kernel for all three roots
    assert _plan([kir.SIN_CHAIN, kir.DSIN_CHAIN, two_x], poly7=True) == "map_chains3"
    # the dedicated pair stays; the other roots are grouped
    assert _plan([kir.SIN_CHAIN, kir.DSIN_CHAIN, two_x, cube]) == "map_sin_dsin_f32,map_chains2"
    # at most 8 roots per kernel
    assert _plan([two_x] * 10) == "map_chains8,map_chains2"
    # two inputs
    ab = kir.chain(E("mul", A, B))
    assert _plan([ab, ab, two_x], n_inputs=2, dtype="f64") == "map_chains3"


def test_roots_that_cannot_share_a_kernel():
    two_x = kir.chain(E("mul", A, C(2.0)))
    # a root that overwrites the input: the next root must see the new values
    mod = kir.map_module([two_x, two_x])
    mod["nodes"][2]["out"] = 0
    m = api.Module(mod)
    assert m.plan([mb.F32] * m.num_buffers) == "map_chain,map_chain"
    # different ranges
    mod = kir.map_module([two_x, two_x])
    for node in mod["nodes"][3:]:
        node["end"] = 100
    m = api.Module(mod)
    assert m.plan([mb.F32] * m.num_buffers) == "map_chain,map_chain"


def test_disk_cache_serves_a_later_process(tmp_path):
    # MLKB_CACHE_DIR: the first process compiles and stores the cubin, a later
    # one loads it without compiling; a file whose stored source differs from
    # the one wanted (a damaged file, or a hash collision) is not used.
    import os
    import subprocess
    import sys

    _nvrtc_or_skip()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("from mlk2_b200 import api, kir\n"
            "ch = kir.chain(kir.E('mul', kir.A, kir.C(0.3)), kir.E('tanh', kir.T(0)))\n"
            "api.chain_build(ch, dtype='f64')\n"
            "print(api.chain_compile(-1)[1])\n")
    cache = tmp_path / "cache"
    env = dict(os.environ, MLKB_CACHE_DIR=str(cache))

    def compiled_in_new_process():
        r = subprocess.run([sys.executable, "-c", code], env=env, cwd=root,
                           capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        return int(r.stdout.strip().splitlines()[-1])

    assert compiled_in_new_process() == 1
    files = list(cache.glob("mlkb-chain-*.cubin"))
    assert len(files) == 1 and files[0].stat().st_size > 1000
    assert compiled_in_new_process() == 0            # loaded from the file
    data = bytearray(files[0].read_bytes())
    data[20] ^= 0xFF                                  # inside the stored source
    files[0].write_bytes(bytes(data))
    assert compiled_in_new_process() == 1            # not trusted: compiled again
    assert compiled_in_new_process() == 0            # and the rewritten file serves


def test_without_nvrtc_chains_are_not_compiled(tmp_path):
    # a process whose NVRTC cannot be loaded: compilation reports inactive,
    # building a chain is refused with the reason, nothing crashes
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import mlk2_b200 as mb\n"
            "from mlk2_b200 import api, kir\n"
            "print(api.chain_compile(-1)[0])\n"
            "try:\n"
            "    api.chain_build(kir.chain(kir.E('mul', kir.A, kir.A)))\n"
            "    print('built')\n"
            "except mb.MLKBError as e:\n"
            "    print('refused', e.status, 'NVRTC' in str(e))\n")
    env = dict(os.environ, MLKB_NVRTC_LIB=str(tmp_path / "libnvrtc-missing.so"))
    r = subprocess.run([sys.executable, "-c", code], env=env, cwd=root, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.strip().splitlines()
    assert lines[-2] == "False"
    assert lines[-1] == f"refused {mb.ERR_UNSUPPORTED} True", lines
