"""Wordle in several scripts as MCP environments (reference environments:
mcp_tools/wordle_multilingual/{core,server_en,server_ja,server_zh}.py).

* ``en``: 5-letter English words; the bundled answer / allowed-guess lists.
* ``ja``: 5-hiragana words; katakana input is folded to hiragana.  The answer is shown with its
  kanji spellings (at most two, ``かんがえる (考える)``).
* ``zh``: 5-symbol zhuyin (bopomofo) spellings without tones, shown with their Chinese words.

The ja / zh dictionaries are JSON objects ``{spelling: [word, ...]}`` — ``answer_dict.json``
(answer pool) and ``valid_dict.json`` (every accepted guess).  The package bundles the
reference's dictionaries (``envs/data/wordle_ja``, ``envs/data/wordle_zh``: 1839 / 1450
answers); ``--data-dir`` points at another pair.  Every guess costs an attempt (invalid ones included); feedback is
``correct`` / ``present`` / ``absent`` per character with duplicates resolved by the two-pass
rule; ``early_exit`` is set when the game ends.

    python -m agent_factory_3_b200.envs.wordle_multilingual --lang ja --seed 3
"""
from __future__ import annotations

import argparse
import json
import random
from pathlib import Path
from typing import Annotated

from .wordle import DATA, MAX_ATTEMPTS, WordleGame, load_words

LANGS = ("en", "ja", "zh")
_KATAKANA0, _KATAKANA1, _SHIFT = 0x30A1, 0x30F6, 0x60  # katakana block -> hiragana


def katakana_to_hiragana(s: str) -> str:
    return "".join(chr(ord(c) - _SHIFT) if _KATAKANA0 <= ord(c) <= _KATAKANA1 else c for c in s)


class GlossedWordleGame(WordleGame):
    """Wordle over spellings that map to words (kana -> kanji, zhuyin -> hanzi)."""

    def __init__(self, answer: str, answers: dict[str, list[str]], valid: dict[str, list[str]],
                 lang: str):
        self.lang = lang
        self.gloss = {**valid, **answers}
        super().__init__(answer, set(valid) | set(answers))

    def normalize(self, word: str) -> str:
        w = word.strip()
        return katakana_to_hiragana(w) if self.lang == "ja" else w

    def display(self, word: str) -> str:
        words = self.gloss.get(word) or []
        return f"{word} ({'/'.join(words[:2])})" if words else word


def load_dict(path: Path) -> dict[str, list[str]]:
    d = json.loads(Path(path).read_text(encoding="utf-8"))
    if not isinstance(d, dict):
        raise ValueError(f"{path}: expected a JSON object of spelling -> [words]")
    return {k: list(v) if isinstance(v, list) else [v] for k, v in d.items()}


_INSTRUCTIONS = {
    "en": "Wordle: guess a 5-letter English word in {n} attempts. Each guess returns per-letter "
          "feedback: 'correct' (right letter, right position), 'present' (in the word, wrong "
          "position), 'absent' (not in the word).",
    "ja": "ひらがな版 Wordle: 5文字のひらがなの単語を{n}回以内に当ててください。各推測の後、文字ごとに "
          "correct（位置も正しい）/ present（別の位置にある）/ absent（含まれない）が返ります。",
    "zh": "注音版 Wordle：在 {n} 次內猜出由 5 個注音符號（不含聲調）組成的詞。每次猜測後，每個符號會得到 "
          "correct（位置正確）/ present（存在但位置不對）/ absent（不存在）的提示。",
}


def make_game(lang: str, data_dir: Path | None = None, target: str | None = None,
              seed: int | None = None) -> WordleGame:
    if lang not in LANGS:
        raise ValueError(f"lang must be one of {LANGS}")
    rng = random.Random(seed)
    if lang == "en":
        answers = sorted(load_words(DATA / "wordle_answers.txt"))
        target = (target or rng.choice(answers)).lower()
        if target not in answers:
            raise ValueError(f"target {target!r} is not in the answers list")
        return WordleGame(target, load_words(DATA / "wordle_allowed.txt") | set(answers))
    if data_dir is None:
        data_dir = DATA / f"wordle_{lang}"
    answers = load_dict(Path(data_dir) / "answer_dict.json")
    valid = load_dict(Path(data_dir) / "valid_dict.json")
    pool = sorted(answers)
    target = target or rng.choice(pool)
    if target not in answers:
        raise ValueError(f"target {target!r} is not in the answers dictionary")
    return GlossedWordleGame(target, answers, valid, lang)


def build_server(lang: str = "en", data_dir: Path | None = None, target: str | None = None,
                 seed: int | None = None):
    from mcp.server.fastmcp import FastMCP

    state = {"game": make_game(lang, data_dir, target, seed)}
    mcp = FastMCP(name=f"WordleGame_{lang}", instructions=_INSTRUCTIONS[lang].format(n=MAX_ATTEMPTS))

    @mcp.tool(description="Make a guess. Returns per-character feedback and the game state.")
    def guess(word: Annotated[str, "the 5-character guess"]) -> dict:
        r = state["game"].guess(word)
        if r.get("game_over"):
            r["early_exit"] = True
        return r

    @mcp.tool(description="Start a new game with a new random answer.")
    def reset_game(seed: Annotated[int | None, "optional random seed"] = None) -> dict:
        state["game"] = make_game(lang, data_dir, None, seed)
        return state["game"].state(message="New game started.")

    mcp.state = state
    return mcp


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--lang", choices=LANGS, default="en")
    ap.add_argument("--data-dir", type=Path, default=None)
    ap.add_argument("--target", default=None)
    ap.add_argument("--seed", type=int, default=None)
    a = ap.parse_args()
    build_server(a.lang, a.data_dir, a.target, a.seed).run()


if __name__ == "__main__":
    main()
