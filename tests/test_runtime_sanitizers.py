"""The C++ host runtime (csrc/runtime/runtime.cpp) under AddressSanitizer + UndefinedBehaviorSanitizer.

The extension is rebuilt with ``-fsanitize=address,undefined`` into a temporary directory and
imported by a child interpreter that preloads the sanitizer runtimes; the child drives every class
through a randomized workload (page allocator churn, decode-metadata rows that allocate pages at
page edges, radix prefix-cache match / insert / release / evict cycles, a shared-memory ring written
by a forked producer and read with wraparound).  Any sanitizer report aborts the child
(``halt_on_error``), so the test passes only with a clean run.  CPU only.
"""
import os
import shutil
import subprocess
import sys
import sysconfig
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _lib(name):
    gcc = shutil.which("gcc")
    if gcc is None:
        return None
    p = subprocess.run([gcc, f"-print-file-name={name}"], capture_output=True, text=True).stdout.strip()
    return p if os.path.isabs(p) and os.path.exists(p) else None


WORKLOAD = textwrap.dedent("""
    import os, random, sys
    import numpy as np
    sys.path.insert(0, sys.argv[1])
    import _runtime as R

    rng = random.Random(7)
    # page allocator churn, including the error paths
    a = R.PageAllocator(512, 1)
    held = []
    for _ in range(2000):
        if held and rng.random() < 0.45:
            a.free(held.pop(rng.randrange(len(held))))
        else:
            n = rng.randint(1, 9)
            if a.can_alloc(n):
                held.append(a.alloc(n))
            else:
                try:
                    a.alloc(n)
                    raise SystemExit("alloc past the pool succeeded")
                except RuntimeError:
                    pass
    for h in held:
        a.free(h)
    assert a.num_free() == 511, a.num_free()

    # decode metadata: requests crossing page edges pull pages from the allocator
    P, PB = 12, 16
    b = R.DecodeMetaBuilder(PB, P)
    out = np.zeros(R.DecodeMetaBuilder.packed_size(PB, P), dtype=np.int32)
    pages = [[] for _ in range(11)]
    lens = [rng.randint(0, 700) for _ in pages]
    for i, n in enumerate(lens):
        pages[i] = a.alloc((n + 63) // 64) if n else []
    for step in range(120):
        kl = np.array(lens, dtype=np.int64)
        n = b.build(out, pages, kl, np.zeros(len(lens), np.int64), np.arange(len(lens), dtype=np.int64),
                    a, PB)
        assert n == len(lens)
        for i in range(len(lens)):
            assert out[i] == lens[i] + 1
            assert out[PB + i] == pages[i][lens[i] // 64] * 64 + lens[i] % 64
        lens = [x + 1 if x + 1 < P * 64 else 0 for x in lens]
        for i, x in enumerate(lens):
            if x == 0:
                a.free(pages[i])
                pages[i] = []
    for pl in pages:
        a.free(pl)

    # prefix cache: shared prefixes, concurrent references, eviction
    pc = R.PrefixCache(64)
    base = [rng.randrange(1000) for _ in range(64 * 6)]
    live = []
    for it in range(300):
        cut = rng.randint(1, 6) * 64
        toks = np.array(base[:cut] + [rng.randrange(1000) for _ in range(rng.randint(0, 200))], dtype=np.int32)
        ns = rng.randrange(2)
        nodes, got = pc.match(ns, toks, len(toks) // 64)
        need = len(toks) // 64 - len(got)
        if not a.can_alloc(need):
            a.free(pc.evict(need))
            if not a.can_alloc(need):
                pc.release(nodes)
                continue
        mine = a.alloc(need) if need else []
        live.append((ns, toks, list(got) + mine, list(nodes)))
        if len(live) > 4 or rng.random() < 0.5:
            ns2, t2, pg2, nd2 = live.pop(rng.randrange(len(live)))
            dup = pc.insert_release(ns2, t2, pg2, nd2)
            a.free(dup)
            own = set(pg2[:len(t2) // 64])
            a.free([p for p in pg2[len(t2) // 64:] if p not in own])
    for ns2, t2, pg2, nd2 in live:
        a.free(pc.insert_release(ns2, t2, pg2, nd2))
    a.free(pc.evict(pc.cached_pages()))
    pc.clear()

    # shared-memory ring: a forked producer, the parent consumes (wraparound, odd sizes)
    name = "/omni_san_%d" % os.getpid()
    ring = R.ShmRing(name, 4096, True)
    msgs = [bytes(rng.randrange(256) for _ in range(rng.randint(1, 900))) for _ in range(200)]
    pid = os.fork()
    if pid == 0:
        w = R.ShmRing(name, 4096, False)
        for m in msgs:
            while not w.put(m):
                pass
        os._exit(0)
    got = []
    while len(got) < len(msgs):
        x = ring.get()
        if x is not None:
            got.append(x)
    os.waitpid(pid, 0)
    assert got == msgs
    print("sanitized workload ok")
""")


@pytest.mark.skipif(shutil.which("g++") is None or _lib("libasan.so") is None or _lib("libubsan.so") is None,
                    reason="needs g++ with the address / undefined sanitizers")
def test_runtime_under_asan_ubsan(tmp_path):
    import pybind11

    so = tmp_path / ("_runtime" + sysconfig.get_config_var("EXT_SUFFIX"))
    cmd = ["g++", "-O1", "-g", "-fsanitize=address,undefined", "-fno-omit-frame-pointer", "-shared", "-fPIC",
           "-std=c++17", f"-I{pybind11.get_include()}", f"-I{sysconfig.get_paths()['include']}",
           os.path.join(ROOT, "csrc", "runtime", "runtime.cpp"), "-o", str(so), "-lrt"]
    subprocess.run(cmd, check=True, timeout=600)
    script = tmp_path / "work.py"
    script.write_text(WORKLOAD)
    env = dict(os.environ,
               LD_PRELOAD=f"{_lib('libasan.so')}:{_lib('libubsan.so')}",
               ASAN_OPTIONS="detect_leaks=0:halt_on_error=1:abort_on_error=1",
               UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
    r = subprocess.run([sys.executable, str(script), str(tmp_path)], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "sanitized workload ok" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])
