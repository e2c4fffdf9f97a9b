"""Wordle as an MCP environment: guess a 5-letter word in 6 attempts; each guess returns
per-letter feedback (correct / present / absent, duplicates resolved with the usual two-pass
rule).  The ``guess`` tool's structured result carries ``early_exit`` once the game is over so
the rollout stops (reference environment: examples/wordle/mcp_tool/server.py).

    python -m agent_factory_3_b200.envs.wordle --target crane
"""
from __future__ import annotations

import argparse
from pathlib import Path
from typing import Annotated

DATA = Path(__file__).parent / "data"
WORD_LENGTH = 5
MAX_ATTEMPTS = 6


def load_words(path: Path) -> set[str]:
    return {ln.strip().lower() for ln in path.read_text().splitlines() if ln.strip()}


def score(guess: str, answer: str) -> list[str]:
    status = ["absent"] * len(guess)
    left: dict[str, int] = {}
    for i, (g, a) in enumerate(zip(guess, answer)):
        if g == a:
            status[i] = "correct"
        else:
            left[a] = left.get(a, 0) + 1
    for i, g in enumerate(guess):
        if status[i] != "correct" and left.get(g, 0) > 0:
            status[i] = "present"
            left[g] -= 1
    return status


class WordleGame:
    """One game.  Words are compared as character sequences of the answer's length, so any
    alphabet works (kana, zhuyin); ``normalize`` and ``display`` are the language hooks."""

    def __init__(self, answer: str, valid: set[str]):
        self.answer = self.normalize(answer)
        self.valid = {self.normalize(w) for w in valid} | {self.answer}
        self.attempts = 0
        self.won = self.lost = False

    def normalize(self, word: str) -> str:
        return word.lower().strip()

    def display(self, word: str) -> str:
        return word

    def state(self, **extra) -> dict:
        out = {"attempts": self.attempts, "attempts_remaining": MAX_ATTEMPTS - self.attempts,
               "won": self.won, "lost": self.lost, "game_over": self.won or self.lost}
        out.update(extra)
        if self.won or self.lost:
            out["answer"] = self.display(self.answer)
        return out

    def guess(self, word: str) -> dict:
        if self.won or self.lost:
            return self.state(error="Game is over.")
        self.attempts += 1
        g = self.normalize(word)
        err = None
        if len(g) != len(self.answer):
            err = f"Word must be exactly {len(self.answer)} letters."
        elif g not in self.valid:
            err = f"'{word}' is not in the allowed word list."
        if err:
            if self.attempts >= MAX_ATTEMPTS:
                self.lost = True
            return self.state(error=err)
        st = score(g, self.answer)
        if g == self.answer:
            self.won = True
        elif self.attempts >= MAX_ATTEMPTS:
            self.lost = True
        return self.state(guess=g, results=[{"char": c, "status": s} for c, s in zip(g, st)])


def build_server(target: str, answers: Path = DATA / "wordle_answers.txt",
                 allowed: Path = DATA / "wordle_allowed.txt"):
    from mcp.server.fastmcp import FastMCP

    ans = load_words(answers)
    if target.lower() not in ans:
        raise ValueError(f"target {target!r} is not in the answers list")
    game = WordleGame(target, load_words(allowed) | ans)
    mcp = FastMCP(name="WordleGame", instructions=(
        f"Wordle: guess a 5-letter English word in {MAX_ATTEMPTS} attempts. Each guess returns "
        "per-letter feedback: 'correct' (right letter, right position), 'present' (in the word, "
        "wrong position), 'absent' (not in the word). Use 'guess' to make a guess. The game ends "
        f"on a win or after {MAX_ATTEMPTS} attempts."))

    @mcp.tool(description="Make a Wordle guess. Returns per-letter feedback and game state.")
    def guess(word: Annotated[str, "The 5-letter word to guess"]) -> dict:
        r = game.guess(word)
        if r.get("game_over"):
            r["early_exit"] = True
        return r

    mcp.game = game
    return mcp


def reward(result, metadata: dict) -> float:
    """1.0 when the last tool step reports a win."""
    for s in reversed(getattr(result, "steps", []) if result is not None else []):
        so = getattr(s, "structured_output", None)
        if so and "won" in so:
            return 1.0 if so["won"] else 0.0
    return 0.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--target", required=True)
    ap.add_argument("--answers", type=Path, default=DATA / "wordle_answers.txt")
    ap.add_argument("--allowed", type=Path, default=DATA / "wordle_allowed.txt")
    a = ap.parse_args()
    build_server(a.target, a.answers, a.allowed).run()


if __name__ == "__main__":
    main()
