"""The module parser behind mlkb_module_create / mlk_bind_module takes any
input without crashing: seeded mutations of valid mlk-kernel modules (keys
dropped, values swapped for other JSON types, huge and negative numbers,
truncated text) and deeply nested input either parse or are rejected with an
error status. Run in a child process, so a crash fails the test cleanly."""
import ast
import os
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = textwrap.dedent('''
    import copy, ctypes as C, json, random, sys
    sys.path.insert(0, sys.argv[1])
    import mlk2_b200 as mb
    from mlk2_b200 import kir
    L = mb.lib()
    seeds = [kir.map_module([kir.SIN_CHAIN]), kir.map_module([kir.SIN_CHAIN, kir.DSIN_CHAIN]),
             kir.call_module("softmax", 5, 7), kir.call_module("matmul", 4, 5, 6),
             kir.qk_softmax_module(256, 64, 0.125)]
    rng = random.Random(20261202)
    vals = [None, True, False, 0, -1, 1, 2**31, 2**63 - 1, -2**63, 1e308, -1e308, 0.5, "",
            "x", [], {}, [1, 2], {"a": 1}]

    def mutate(o):
        if isinstance(o, dict) and o:
            k = rng.choice(list(o))
            r = rng.random()
            if r < 0.2:
                del o[k]
            elif r < 0.5:
                o[k] = copy.deepcopy(rng.choice(vals))
            else:
                mutate(o[k])
        elif isinstance(o, list) and o:
            i = rng.randrange(len(o))
            r = rng.random()
            if r < 0.2:
                del o[i]
            elif r < 0.35:
                o.append(copy.deepcopy(o[i]))
            elif r < 0.6:
                o[i] = copy.deepcopy(rng.choice(vals))
            else:
                mutate(o[i])

    seen = set()
    texts = ["[" * 200000, '{"a":' * 100000 + "1" + "}" * 100000]
    for _ in range(1500):
        m = copy.deepcopy(rng.choice(seeds))
        for _ in range(rng.randint(1, 4)):
            mutate(m)
        t = json.dumps(m)
        texts.append(t[:rng.randrange(len(t) + 1)] if rng.random() < 0.2 else t)
    for t in texts:
        h = C.c_void_p()
        st = L.mlkb_module_create(t.encode(), C.byref(h))
        seen.add(st)
        if st == 0 and h.value:
            L.mlkb_module_kind(h)
            L.mlkb_module_num_buffers(h)
            L.mlkb_module_destroy(h)
        L.mlk_bind_module(t.encode())
    L.mlk_bind_module(None)
    print("statuses", sorted(seen))
''')


def test_parser_survives_mutated_and_nested_input():
    r = subprocess.run([sys.executable, "-c", _CHILD, ROOT], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, (r.returncode, r.stderr[-2000:])
    statuses = ast.literal_eval(r.stdout.strip().split("statuses", 1)[1].strip())
    assert 0 in statuses and any(s != 0 for s in statuses)
