"""Concurrency stress test of the Python tool sandbox (the reference runs one against its MCP
server: ``mcp_tools/python_tool/stress_test.py:131-190``).

Every simulated rollout is one session that runs a short multi-step problem: each step's code
depends on the state the earlier steps left in the session, and each step's output is checked
against the value computed here, so a lost, mixed-up or restarted session counts as an error.
Rollouts run ``concurrency`` at a time, either against an in-process ``SessionPool`` (default) or
against a running MCP server (``--url``, streamable HTTP, tools ``run_python`` /
``reset_session``).  The report gives successes, grouped errors, steps, wall time, rollouts per
second and per-rollout latency percentiles.

    python -m agent_factory_3_b200.envs.sandbox_stress --sessions 64 --concurrency 16 --seccomp
    python -m agent_factory_3_b200.envs.sandbox_stress --url http://127.0.0.1:8811/mcp
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field


@dataclass
class Problem:
    steps: list[str]            # code cells, run in order in one session
    expect: list[str]           # substring each step's stdout must contain


def make_problem(rng: random.Random) -> Problem:
    """One of a few stateful multi-step problems with known answers (stdlib only)."""
    kind = rng.randrange(4)
    if kind == 0:       # quadratic with integer roots: solve, verify, sum
        r1, r2 = rng.randint(-20, 20), rng.randint(-20, 20)
        b, c = -(r1 + r2), r1 * r2
        return Problem(
            [f"import math\nb, c = {b}, {c}\nd = b*b - 4*c\nroots = sorted([(-b - math.isqrt(d))//2, "
             f"(-b + math.isqrt(d))//2])\nprint('roots', roots)",
             "print('verify', all(r*r + b*r + c == 0 for r in roots))",
             "print('sum', sum(roots))"],
            [f"roots {sorted([r1, r2])}", "verify True", f"sum {r1 + r2}"])
    if kind == 1:       # number theory across steps
        n = rng.randint(10_000, 2_000_000)
        fac: dict[int, int] = {}
        m, p = n, 2
        while p * p <= m:
            while m % p == 0:
                fac[p] = fac.get(p, 0) + 1
                m //= p
            p += 1
        if m > 1:
            fac[m] = fac.get(m, 0) + 1
        return Problem(
            [f"n = {n}\nf = {{}}\nm, p = n, 2\nwhile p * p <= m:\n    while m % p == 0:\n"
             f"        f[p] = f.get(p, 0) + 1\n        m //= p\n    p += 1\nif m > 1:\n"
             f"    f[m] = f.get(m, 0) + 1\nprint('nf', len(f))",
             "import math\nprint('prod', math.prod(k ** v for k, v in f.items()) == n)",
             "print('largest', max(f))"],
            [f"nf {len(fac)}", "prod True", f"largest {max(fac)}"])
    if kind == 2:       # fractions: harmonic partial sums
        k = rng.randint(5, 40)
        from fractions import Fraction
        h = sum(Fraction(1, i) for i in range(1, k + 1))
        return Problem(
            [f"from fractions import Fraction\nk = {k}\nh = sum(Fraction(1, i) for i in range(1, k + 1))",
             "print('den', h.denominator)",
             "print('num_mod', h.numerator % 1000003)"],
            ["", f"den {h.denominator}", f"num_mod {h.numerator % 1000003}"])
    # kind 3: a CPU-heavier step (sieve) then queries on its result
    n = rng.randint(20_000, 200_000)
    sieve = bytearray([1]) * (n + 1)
    sieve[0:2] = b"\x00\x00"
    for i in range(2, int(n ** 0.5) + 1):
        if sieve[i]:
            sieve[i * i::i] = bytearray(len(sieve[i * i::i]))
    primes = [i for i in range(n + 1) if sieve[i]]
    return Problem(
        [f"n = {n}\ns = bytearray([1]) * (n + 1)\ns[0:2] = b'\\x00\\x00'\n"
         f"for i in range(2, int(n ** 0.5) + 1):\n    if s[i]:\n"
         f"        s[i*i::i] = bytearray(len(s[i*i::i]))\nprimes = [i for i in range(n + 1) if s[i]]\n"
         f"print('count', len(primes))",
         "print('last', primes[-1])",
         "print('twin', sum(1 for a, b in zip(primes, primes[1:]) if b - a == 2))"],
        [f"count {len(primes)}", f"last {primes[-1]}",
         f"twin {sum(1 for a, b in zip(primes, primes[1:]) if b - a == 2)}"])


@dataclass
class Report:
    total: int = 0
    success: int = 0
    steps: int = 0
    errors: list[tuple[int, str]] = field(default_factory=list)
    latency: list[float] = field(default_factory=list)
    wall_s: float = 0.0

    def summary(self) -> dict:
        el = sorted(self.latency)

        def pct(q):
            return round(el[min(len(el) - 1, int(len(el) * q))], 3) if el else None
        groups: dict[str, int] = {}
        for _, e in self.errors:
            groups[e[:80]] = groups.get(e[:80], 0) + 1
        return {"total": self.total, "success": self.success, "errors": len(self.errors),
                "steps": self.steps, "wall_s": round(self.wall_s, 2),
                "rollouts_per_s": round(self.total / self.wall_s, 2) if self.wall_s else None,
                "latency_s": {"p50": pct(0.5), "p90": pct(0.9), "p99": pct(0.99),
                              "max": round(el[-1], 3) if el else None},
                "success_rate": round(self.success / max(1, self.total), 4),
                "error_breakdown": dict(sorted(groups.items(), key=lambda kv: -kv[1])[:10])}


def _check(problem: Problem, outputs: list[dict]) -> str | None:
    for i, (want, out) in enumerate(zip(problem.expect, outputs)):
        if not out.get("ok"):
            return f"step {i} failed: {(out.get('stderr') or '')[-160:]}"
        if want and want not in out.get("stdout", ""):
            return f"step {i}: expected {want!r}, got {out.get('stdout', '')[:80]!r}"
    return None


def run_local(sessions: int, concurrency: int, seed: int = 0, **session_kw) -> Report:
    """Rollouts against an in-process session pool, ``concurrency`` threads at a time."""
    from .python_sandbox import SessionPool
    pool = SessionPool(**session_kw)
    rep = Report()
    rng = random.Random(seed)
    problems = [make_problem(rng) for _ in range(sessions)]

    def one(idx: int):
        t0 = time.monotonic()
        name = f"stress-{idx}"
        sess = pool.get(name)
        outs = []
        try:
            for code in problems[idx].steps:
                outs.append(sess.run(code))
            err = _check(problems[idx], outs)
        except Exception as e:  # noqa: BLE001
            err = f"{type(e).__name__}: {e}"
        finally:
            sess.stop()
        return idx, err, len(outs), time.monotonic() - t0

    t0 = time.monotonic()
    try:
        with ThreadPoolExecutor(max_workers=concurrency) as ex:
            for idx, err, n, dt in ex.map(one, range(sessions)):
                rep.total += 1
                rep.steps += n
                rep.latency.append(dt)
                if err:
                    rep.errors.append((idx, err))
                else:
                    rep.success += 1
    finally:
        pool.close()
    rep.wall_s = time.monotonic() - t0
    return rep


async def run_remote(url: str, sessions: int, concurrency: int, seed: int = 0,
                     timeout: float = 60.0) -> Report:
    """Rollouts against a running MCP python server (one client connection per rollout)."""
    from ..rollout.mcp_client import McpClient
    rep = Report()
    rng = random.Random(seed)
    problems = [make_problem(rng) for _ in range(sessions)]
    sem = asyncio.Semaphore(concurrency)

    async def one(idx: int):
        async with sem:
            t0 = time.monotonic()
            outs, err = [], None
            name = f"stress-{idx}-{seed}"
            try:
                async with McpClient({"url": url}) as c:
                    for code in problems[idx].steps:
                        r = await c.call_tool("run_python", {"code": code, "session": name},
                                              timeout=timeout)
                        payload = getattr(r, "structuredContent", None)
                        if not payload:
                            text = "".join(getattr(b, "text", "") for b in r.content)
                            payload = json.loads(text) if text.startswith("{") else {"ok": False, "stderr": text}
                        outs.append(payload.get("result", payload)
                                    if "ok" not in payload else payload)
                    await c.call_tool("reset_session", {"session": name}, timeout=timeout)
                err = _check(problems[idx], outs)
            except Exception as e:  # noqa: BLE001
                err = f"{type(e).__name__}: {e}"
            rep.total += 1
            rep.steps += len(outs)
            rep.latency.append(time.monotonic() - t0)
            if err:
                rep.errors.append((idx, err))
            else:
                rep.success += 1

    t0 = time.monotonic()
    await asyncio.gather(*(one(i) for i in range(sessions)))
    rep.wall_s = time.monotonic() - t0
    return rep


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--concurrency", type=int, default=16)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--url", default=None, help="MCP python server (streamable HTTP) to stress")
    ap.add_argument("--seccomp", action="store_true", help="(local) lock workers with seccomp")
    ap.add_argument("--timeout", type=float, default=30.0)
    a = ap.parse_args()
    if a.url:
        rep = asyncio.run(run_remote(a.url, a.sessions, a.concurrency, a.seed, a.timeout))
    else:
        rep = run_local(a.sessions, a.concurrency, a.seed, timeout=a.timeout,
                        use_seccomp=a.seccomp, use_bwrap=False)
    print(json.dumps(rep.summary(), indent=1))


if __name__ == "__main__":
    main()
