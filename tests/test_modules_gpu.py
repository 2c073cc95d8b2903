"""Module-level paths on the GPU: the poly7 sine family, modules compiled by
the reference's own pipeline, scalar tables of any size and roots with their
own static ranges -- each against the reference's results.

Bars: f32 maps <= 2 ULP of the f64 reference rounded to f32; the poly7 family
bit-exact (it is restated in the same IEEE operations); f64 arithmetic
bit-exact; f64 transcendentals <= 4 / 8 f64 ULP (CUDA vs glibc libm).
"""
import json

import numpy as np
import pytest

import mlk2_b200 as mb
import oracle
from mlk2_b200 import api, kir
from tests.gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu


def same_bits(a, b):
    """Bit-identical, except that any NaN matches any NaN: the encoding of a
    NaN an invalid operation creates differs between the reference's x86-64
    host (negative quiet NaN) and the GPU (its canonical NaN)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    na, nb = np.isnan(a), np.isnan(b)
    if a.shape != b.shape or not np.array_equal(na, nb):
        return False
    bad = np.flatnonzero(a[~na].view(np.int64) != b[~nb].view(np.int64))
    assert bad.size == 0, (a[~na][bad[:5]], b[~nb][bad[:5]])
    return True


def test_poly7_bit_exact(cuda, golden, chain_path):
    g = golden("map_poly7")
    # f64 inputs, f64 outputs: bit for bit (NaN as a class)
    x = dev(cuda, g["x"])
    y = empty(cuda, x.shape, cuda.float64)
    api.map_chain(g["chain_sin"], x, y, poly7=True)
    assert same_bits(host(y), g["sin"])
    # f32 inputs: the same f64 value rounded once, so 0 ULP
    xf = dev(cuda, g["xf"])
    for ch, key in ((g["chain_sin"], "sin_f"), (g["chain_u"], "sin_u_f")):
        yf = empty(cuda, xf.shape, cuda.float32)
        api.map_chain(ch, xf, yf, poly7=True)
        assert oracle.ulp_f32(host(yf), g[key]).max() == 0, key
    # through a module (family="poly7" on the Compute node)
    m = api.Module(kir.map_module([kir.SIN_CHAIN], poly7=True))
    assert m.plan([mb.F32, mb.F32]) == "map_chain_poly7"
    yf = empty(cuda, xf.shape, cuda.float32)
    m.run_dev([xf, yf], n=xf.numel())
    assert oracle.ulp_f32(host(yf), g["sin_u_f"]).max() == 0


def test_poly7_reference_abi(cuda, golden):
    g = golden("map_poly7")
    x = np.ascontiguousarray(g["x"])
    y = np.zeros_like(x)
    assert api.legacy_call(kir.map_module([g["chain_sin"]], poly7=True, dtype="f64"),
                           [x, y], x.size) == 0
    assert same_bits(y, g["sin"])


def _pipeline(golden):
    g = golden("pipeline")
    return g, {k: json.loads(str(g[k + "_json"])) for k in ("sin", "dsin", "both", "scalar")}


def test_pipeline_modules_f32(cuda, golden):
    # The reference's Tier-1 output for y and its calculus-pass derivative,
    # as one two-root module: the dedicated fused kernel runs it.
    g, m = _pipeline(golden)
    both = api.Module(m["both"])
    assert both.plan([mb.F32] * 3) == "map_sin_dsin_f32"
    x = dev(cuda, g["x"])
    y = empty(cuda, x.shape, cuda.float32)
    dy = empty(cuda, x.shape, cuda.float32)
    both.run_dev([x, y, dy], n=0)   # static bounds: n is not read
    assert oracle.ulp_f32(host(y), g["y"]).max() <= 2
    assert oracle.ulp_f32(host(dy), g["dy"]).max() <= 2
    # host buffers, the caller's device and every visible device
    for n_gpus in (1, 0):
        yh, dyh = np.full(g["x"].size, np.nan, np.float32), np.full(g["x"].size, np.nan, np.float32)
        both.run_host([g["x"], yh, dyh], n=0, n_gpus=n_gpus)
        assert oracle.ulp_f32(yh, g["y"]).max() <= 2
        assert oracle.ulp_f32(dyh, g["dy"]).max() <= 2
    # the derivative on its own takes the generic chain, to the same bar
    d = api.Module(m["dsin"])
    dy2 = empty(cuda, x.shape, cuda.float32)
    d.run_dev([x, dy2])
    assert oracle.ulp_f32(host(dy2), g["dy"]).max() <= 2


def test_pipeline_modules_reference_abi(cuda, golden):
    g, m = _pipeline(golden)
    x = g["x"].astype(np.float64)
    y, dy = np.zeros_like(x), np.zeros_like(x)
    assert api.legacy_call(m["both"], [x, y, dy], x.size) == 0
    assert oracle.ulp_f64(y, g["y"]).max() <= 4
    assert oracle.ulp_f64(dy, g["dy"]).max() <= 8
    # the scalar form: x arrives as ScalarParam 0, one output element
    for v, want in zip(g["scalar_x"], g["scalar_y"]):
        out = np.zeros(1)
        assert api.legacy_call(m["scalar"], [out], 1, scalars=[v]) == 0
        assert oracle.ulp_f64(out, np.array([want])).max() <= 4


def test_scalar_table_of_any_size(cuda, chain_path):
    # ScalarParam 100 of a 150-entry table, and 200 past its end (reads 0)
    ch = kir.chain(kir.E("mul", kir.A, kir.S(100)), kir.E("add", kir.T(0), kir.S(5)),
                   kir.E("add", kir.T(1), kir.S(200)))
    scalars = np.arange(150, dtype=np.float64) * 0.75 - 3.0
    xh = np.linspace(-5, 5, 1000)
    x = dev(cuda, xh)
    y = empty(cuda, x.shape, cuda.float64)
    api.map_chain(ch, x, y, scalars=list(scalars))
    (want,) = oracle.port().chain([ch], xh, scalars=scalars)
    assert same_bits(host(y), want)
    # and through the reference ABI, where the driver passes the whole table
    yh = np.zeros_like(xh)
    assert api.legacy_call(kir.map_module([ch], dtype="f64"), [xh.copy(), yh], xh.size,
                           scalars=list(scalars)) == 0
    assert same_bits(yh, want)


def test_roots_with_their_own_static_ranges(cuda):
    # root 0 stores [0, 1000) whatever n is; root 1 runs to the caller's n;
    # each buffer is exactly as long as its root's range, so a copy past it
    # would write outside the caller's array
    mod = kir.map_module([kir.SIN_CHAIN, kir.chain(kir.E("mul", kir.A, kir.C(2.0)))])
    mod["nodes"][0]["end"] = 1000
    m = api.Module(mod)
    xh = np.linspace(-3, 3, 1000).astype(np.float32)
    y0 = np.full(1000, np.nan, np.float32)
    y1 = np.full(500, np.nan, np.float32)
    m.run_host([xh, y0, y1], n=500, n_gpus=1)
    (r0,) = oracle.port().chain([kir.SIN_CHAIN], xh.astype(np.float64))
    assert oracle.ulp_f32(y0, r0).max() <= 2
    assert np.array_equal(y1, xh[:500] * 2)


def _wide_chain(live):
    """`live` products of x kept alive at once, then summed: needs `live` + 1
    register slots (or the local-array interpreter past 8)."""
    A, C, T, E = kir.A, kir.C, kir.T, kir.E
    ex = [E("mul", A, C(1.0 + 0.5 * j)) for j in range(live)]
    acc = len(ex)
    ex.append(E("add", T(0), T(1)))
    for j in range(2, live):
        ex.append(E("add", T(len(ex) - 1), T(j)))
    ex.append(E("mul", T(len(ex) - 1), A))        # reads x once more
    ex.append(E("exp", C(0.0)))                    # a dead result (never read)
    ex.append(E("sub", T(len(ex) - 2), C(0.25)))
    return kir.chain(*ex)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("live", [2, 6, 11])
def test_chain_slot_allocation_paths(cuda, dtype, live, chain_path):
    # 2 live temps: 4 register slots; 6: 8 slots; 11: the local-array
    # interpreter. Arithmetic chains are bit-exact in f64 and round once to
    # f32, so both dtypes must equal the oracle exactly.
    ch = _wide_chain(live)
    xh = np.linspace(-3, 3, 100003).astype(dtype)
    (want,) = oracle.port().chain([ch], xh.astype(np.float64))
    for off in (0, 1):                               # 1: unaligned -> the fallback
        x = dev(cuda, xh)[off:]
        y = empty(cuda, (xh.size,), cuda.float64 if dtype == np.float64 else cuda.float32)[off:]
        api.map_chain(ch, x, y)
        got = host(y).astype(np.float64)
        assert np.array_equal(got, want[off:].astype(dtype).astype(np.float64)), (live, off)


def test_chain_two_inputs_and_tail(cuda, chain_path):
    # ElemA and ElemB through the staged loads, lengths around a tile edge
    ch = kir.chain(kir.E("mul", kir.A, kir.B), kir.E("div", kir.T(0), kir.B),
                   kir.E("add", kir.T(1), kir.A))
    for n in (1, 4, 1023, 1024, 1025, 4096 * 3 + 3):
        rng = np.random.default_rng(n)
        ah = rng.normal(0, 2, n)
        bh = rng.normal(0, 2, n)
        bh[::7] = 0.0                                 # Div by 0 -> 0
        y = empty(cuda, (n,), cuda.float64)
        api.map_chain(ch, dev(cuda, ah), y, b=dev(cuda, bh))
        (want,) = oracle.port().chain([ch], ah, bh)
        assert np.array_equal(host(y), want), n


def test_compiled_chain_reused_across_constants_and_scalars(cuda):
    # one compiled kernel per chain structure: other constant or scalar values
    # reuse it, and each call still computes with its own values
    api.chain_compile(1)
    xh = np.linspace(-4, 4, 4099)
    x = dev(cuda, xh)
    _, c0, _ = api.chain_compile(-1)
    for v in (0.5, 3.0, -1.25):
        ch = kir.chain(kir.E("mul", kir.A, kir.C(v)), kir.E("add", kir.T(0), kir.S(1)))
        y = empty(cuda, x.shape, cuda.float64)
        api.map_chain(ch, x, y, scalars=[0.0, 2 * v])
        (want,) = oracle.port().chain([ch], xh, scalars=[0.0, 2 * v])
        assert same_bits(host(y), want), v
    _, c1, _ = api.chain_compile(-1)
    assert c1 - c0 <= 1, (c0, c1)


@pytest.mark.parametrize("dtype", ["f32", "f64"])
def test_root_group_runs_as_one_kernel(cuda, dtype, chain_path):
    # four roots no dedicated kernel matches (the poly7 family), one input:
    # compiled, ONE kernel writes all four outputs, each bit-identical to the
    # root run on its own; interpreted, the roots run one by one (the counter
    # counts compiled launches only)
    E, A, C, T = kir.E, kir.A, kir.C, kir.T
    chains = [kir.SIN_CHAIN, kir.DSIN_CHAIN, kir.chain(E("mul", A, C(2.0))),
              kir.chain(E("mul", A, A), E("mul", T(0), A))]
    m = api.Module(kir.map_module(chains, poly7=True, dtype=dtype))
    tdt = cuda.float32 if dtype == "f32" else cuda.float64
    assert m.plan([mb.F32 if dtype == "f32" else mb.F64] * m.num_buffers) == "map_chains4"
    n = 100003
    x = dev(cuda, np.linspace(-7.0, 7.0, n).astype(np.float32 if dtype == "f32" else np.float64))
    outs = [empty(cuda, (n,), tdt) for _ in chains]
    _, _, before = api.chain_compile(-1)
    m.run_dev([x] + outs, n=n)
    cuda.cuda.synchronize()
    _, _, after = api.chain_compile(-1)
    assert after - before == (1 if chain_path == "compiled" else 0)  # compiled launches
    for ch, o in zip(chains, outs):
        want = empty(cuda, (n,), tdt)
        api.map_chain(ch, x, want, poly7=True)
        assert same_bits(host(o), host(want))


def test_two_input_group_through_the_reference_abi(cuda):
    # f64 host buffers through mlk_kernel; the roots share x and w, one root
    # reads only x; arithmetic chains are bit-exact against the executor
    E, A, B, C, T = kir.E, kir.A, kir.B, kir.C, kir.T
    chains = [kir.chain(E("mul", A, B)), kir.chain(E("mul", A, B), E("sub", T(0), A)),
              kir.chain(E("mul", A, C(2.0)))]
    mod = kir.map_module(chains, n_inputs=2, dtype="f64")
    assert api.Module(mod).plan([mb.F64] * 5) == "map_chains3"
    n = 70001
    rng = np.random.default_rng(11)
    x, w = rng.normal(0, 3, n), rng.normal(0, 3, n)
    outs = [np.zeros(n) for _ in chains]
    assert api.legacy_call(mod, [x, w] + outs, n) == 0
    for ch, o in zip(chains, outs):
        (want,) = oracle.port().chain([ch], x, w)
        assert np.array_equal(o, want)


def test_f32_chain_cancelling_after_sin_and_cos(cuda, chain_path):
    # sin(x) - sin(pi/4) and cos(x) - cos(pi/4) for f32 x around pi/4: the
    # results are tiny, so any error of sin / cos beyond f64 accuracy would
    # show as many f32 ULPs; the reference's libm is accurate to an f64 ulp
    E, A, C, T = kir.E, kir.A, kir.C, kir.T
    xh = np.linspace(0.78, 0.79, 20011).astype(np.float32)
    x = dev(cuda, xh)
    for op in ("sin", "cos"):
        ch = kir.chain(E(op, A), E("sub", T(0), C(0.7071067811865476)))
        y = empty(cuda, x.shape, cuda.float32)
        api.map_chain(ch, x, y)
        (want,) = oracle.port().chain([ch], xh.astype(np.float64))
        assert oracle.ulp_f32(host(y), want).max() <= 2, op


def test_chain_loaded_from_the_disk_cache_runs(cuda, tmp_path):
    # two processes with the same MLKB_CACHE_DIR: the first compiles, the
    # second loads the stored cubin; both run the chain to the same bits
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import sys, numpy as np, torch\n"
            "from mlk2_b200 import api, kir\n"
            "ch = kir.chain(kir.E('mul', kir.A, kir.C(0.3)), kir.E('cos', kir.T(0)),\n"
            "               kir.E('add', kir.T(1), kir.A))\n"
            "x = torch.linspace(-50, 50, 100003, device='cuda')\n"
            "y = torch.empty_like(x)\n"
            "api.map_chain(ch, x, y)\n"
            "np.save(sys.argv[1], y.cpu().numpy())\n"
            "print(api.chain_compile(-1)[1])\n")
    env = dict(os.environ, MLKB_CACHE_DIR=str(tmp_path / "cache"))
    outs, compiled = [], []
    for i in range(2):
        path = str(tmp_path / f"y{i}.npy")
        r = subprocess.run([sys.executable, "-c", code, path], env=env, cwd=root,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        compiled.append(int(r.stdout.strip().splitlines()[-1]))
        outs.append(np.load(path))
    assert compiled == [1, 0]
    assert np.array_equal(outs[0].view(np.int32), outs[1].view(np.int32))


def test_process_without_nvrtc_gives_the_same_bits(cuda, tmp_path):
    # the same module and inputs in a process that can load NVRTC (compiled
    # chains, one kernel for the root group) and in one that cannot (the
    # interpreter, root by root): identical outputs
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import sys, numpy as np, torch\n"
            "import mlk2_b200 as mb\n"
            "from mlk2_b200 import api, kir\n"
            "E, A, C, T = kir.E, kir.A, kir.C, kir.T\n"
            "chains = [kir.SIN_CHAIN, kir.DSIN_CHAIN, kir.chain(E('exp', A), E('mul', T(0), C(0.5)))]\n"
            "m = api.Module(kir.map_module(chains, poly7=True))\n"
            "x = torch.linspace(-9, 9, 65537, device='cuda')\n"
            "ys = [torch.empty_like(x) for _ in chains]\n"
            "m.run_dev([x] + ys, n=x.numel())\n"
            "np.save(sys.argv[1], torch.stack(ys).cpu().numpy())\n"
            "print(api.chain_compile(-1)[0], m.plan([mb.F32] * 4))\n")
    outs, info = [], []
    for i, lib in enumerate((None, str(tmp_path / "libnvrtc-missing.so"))):
        env = dict(os.environ)
        if lib is not None:
            env["MLKB_NVRTC_LIB"] = lib
        path = str(tmp_path / f"y{i}.npy")
        r = subprocess.run([sys.executable, "-c", code, path], env=env, cwd=root,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        info.append(r.stdout.strip().splitlines()[-1])
        outs.append(np.load(path))
    assert info == ["True map_chains3", "False map_chains3"]
    assert np.array_equal(outs[0].view(np.int32), outs[1].view(np.int32))


def test_root_group_with_a_large_constant_block(cuda):
    # 8 roots x 40 expressions with 80 distinct constants each: 640 constants
    # (5 KB) in one kernel's parameter block; each output as its root alone
    E, A, C, T = kir.E, kir.A, kir.C, kir.T
    chains = []
    for r in range(8):
        ex = [E("mul", A, C(1.0 + r / 8))]
        for k in range(39):
            op = "add" if k % 2 == 0 else "mul"
            ex.append(E(op, T(len(ex) - 1), C(0.5 + 0.01 * (r * 40 + k))))
        chains.append(kir.chain(*ex))
    m = api.Module(kir.map_module(chains, dtype="f64"))
    assert m.plan([mb.F64] * m.num_buffers) == "map_chains8"
    n = 10007
    x = dev(cuda, np.linspace(-1.0, 1.0, n))
    outs = [empty(cuda, (n,), cuda.float64) for _ in chains]
    api.chain_compile(1)
    m.run_dev([x] + outs, n=n)
    for ch, o in zip(chains, outs):
        want = empty(cuda, (n,), cuda.float64)
        api.map_chain(ch, x, want)
        assert same_bits(host(o), host(want))
