"""Minesweeper as an MCP environment (reference environment: examples/minesweeper/mcp_tool/
core.py:22-470 and server.py:14-170).

* Mines are placed on the first reveal, never on the clicked cell or its neighbours (when the
  board leaves room), so the first click always opens an area.
* ``no_guess=True`` redraws the mine layout until a logic-only solver clears the board from the
  first click: repeated single-cell rules (a number whose remaining mines equal its hidden
  neighbours, or are already all flagged) and pairwise subset rules between two numbers'
  hidden-neighbour sets.  After ``no_guess_max_attempts`` draws the last layout is kept.
* Board text: ``.`` hidden, ``F`` flagged, ``_`` empty, ``1``-``8`` counts, ``*`` mine (shown
  when the game ends).  JSON mode adds row/column coordinates; text mode returns the bare grid
  plus a status line and ``(text, metadata)``.  ``early_exit`` is set once the game ends.

    python -m agent_factory_3_b200.envs.minesweeper --width 9 --height 9 --mines 10 --seed 1
"""
from __future__ import annotations

import argparse
import random
from typing import Annotated


def neighbours(x: int, y: int, w: int, h: int):
    for dy in (-1, 0, 1):
        for dx in (-1, 0, 1):
            if (dx or dy) and 0 <= x + dx < w and 0 <= y + dy < h:
                yield x + dx, y + dy


def solvable_without_guessing(w: int, h: int, mines: set, start: tuple[int, int]) -> bool:
    """True when deductions alone (single-cell and subset rules) open every safe cell."""
    counts = {(x, y): sum((n in mines) for n in neighbours(x, y, w, h))
              for y in range(h) for x in range(w) if (x, y) not in mines}
    opened: set = set()
    known_mines: set = set()

    def open_cell(c):
        stack = [c]
        while stack:
            cur = stack.pop()
            if cur in opened:
                continue
            opened.add(cur)
            if counts[cur] == 0:
                stack.extend(n for n in neighbours(*cur, w, h) if n not in opened)

    open_cell(start)
    total = len(counts)
    while len(opened) < total:
        changed = False
        constraints = []
        for c in list(opened):
            if counts[c] == 0:
                continue
            hidden = [n for n in neighbours(*c, w, h) if n not in opened and n not in known_mines]
            if not hidden:
                continue
            need = counts[c] - sum(n in known_mines for n in neighbours(*c, w, h))
            if need == 0:
                for n in hidden:
                    open_cell(n)
                changed = True
            elif need == len(hidden):
                known_mines.update(hidden)
                changed = True
            else:
                constraints.append((frozenset(hidden), need))
        if changed:
            continue
        for a, na in constraints:           # subset rule: B within A -> A\B holds na-nb mines
            for b, nb in constraints:
                if a is b or not b < a:
                    continue
                rest = a - b
                if na - nb == 0:
                    for n in rest:
                        open_cell(n)
                    changed = True
                elif na - nb == len(rest):
                    known_mines.update(rest)
                    changed = True
        if not changed:
            return False
    return True


class MinesweeperGame:
    def __init__(self, width: int = 9, height: int = 9, num_mines: int = 10, seed: int | None = None,
                 text_mode: bool = False, no_guess: bool = True, no_guess_max_attempts: int = 5000):
        if width < 1 or height < 1:
            raise ValueError("width and height must be at least 1")
        if not 0 <= num_mines < width * height:
            raise ValueError("number of mines must be in [0, width*height)")
        self.width, self.height, self.num_mines = width, height, num_mines
        self.rng = random.Random(seed)
        self.text_mode = text_mode
        self.no_guess = no_guess
        self.no_guess_max_attempts = no_guess_max_attempts
        self.reset()

    def reset(self, seed: int | None = None) -> None:
        if seed is not None:
            self.rng = random.Random(seed)
        self.mines: set = set()
        self.opened: set = set()
        self.flags: set = set()
        self.state = "playing"
        self.placed = False
        self.layout_attempts = 0

    # ------------------------------------------------------------------ board
    def _count(self, c) -> int:
        return sum((n in self.mines) for n in neighbours(*c, self.width, self.height))

    def _place(self, first: tuple[int, int]) -> None:
        cells = [(x, y) for y in range(self.height) for x in range(self.width)]
        keep_out = {first, *neighbours(*first, self.width, self.height)}
        pool = [c for c in cells if c not in keep_out]
        if len(pool) < self.num_mines:
            pool = [c for c in cells if c != first]
        tries = self.no_guess_max_attempts if self.no_guess else 1
        for i in range(max(1, tries)):
            mines = set(self.rng.sample(pool, self.num_mines))
            self.layout_attempts = i + 1
            if not self.no_guess or solvable_without_guessing(self.width, self.height, mines, first):
                break
        self.mines = mines
        self.placed = True

    def _open(self, c) -> int:
        n0 = len(self.opened)
        stack = [c]
        while stack:
            cur = stack.pop()
            if cur in self.opened or cur in self.flags:
                continue
            self.opened.add(cur)
            if self._count(cur) == 0:
                stack.extend(n for n in neighbours(*cur, self.width, self.height) if n not in self.opened)
        return len(self.opened) - n0

    def render(self, reveal_all: bool = False, coords: bool = True) -> str:
        cw = len(str(self.width - 1))
        rows = ["   " + " ".join(str(i).rjust(cw) for i in range(self.width))] if coords else []
        for y in range(self.height):
            cells = []
            for x in range(self.width):
                c = (x, y)
                if reveal_all or c in self.opened:
                    cells.append("*" if c in self.mines else (str(self._count(c)) if self._count(c) else "_"))
                else:
                    cells.append("F" if c in self.flags else ".")
            rows.append((str(y).rjust(2) + " " + " ".join(s.rjust(cw) for s in cells)) if coords
                        else " ".join(cells))
        return "\n".join(rows)

    # ------------------------------------------------------------------ actions
    def _check(self, x: int, y: int, action: str):
        if not (0 <= x < self.width and 0 <= y < self.height):
            return self._respond(error=f"Coordinates ({x}, {y}) out of bounds. Valid range: "
                                       f"x=0-{self.width - 1}, y=0-{self.height - 1}",
                                 action=(action, x, y, "error: out of bounds"))
        if self.state != "playing":
            return self._respond(error=f"Game is over ({self.state}). Use reset_game to start a new game.",
                                 action=(action, x, y, "error: game over"))
        return None

    def reveal(self, x: int, y: int):
        bad = self._check(x, y, "reveal")
        if bad is not None:
            return bad
        c = (x, y)
        if c in self.flags:
            return self._respond(error=f"Cell ({x}, {y}) is flagged. Remove flag first.",
                                 action=("reveal", x, y, "error: cell flagged"))
        if c in self.opened:
            return self._respond(error=f"Cell ({x}, {y}) is already revealed.",
                                 action=("reveal", x, y, "error: already revealed"))
        if not self.placed:
            self._place(c)
        if c in self.mines:
            self.state = "lost"
            return self._respond(message="BOOM! You hit a mine!", action=("reveal", x, y, "BOOM!"))
        n = self._open(c)
        if len(self.opened) == self.width * self.height - self.num_mines:
            self.state = "won"
            return self._respond(message="Congratulations! You won!",
                                 action=("reveal", x, y, f"WIN! opened {n} cells"))
        return self._respond(action=("reveal", x, y, f"opened {n} cells"))

    def toggle_flag(self, x: int, y: int):
        bad = self._check(x, y, "flag")
        if bad is not None:
            return bad
        c = (x, y)
        if c in self.opened:
            return self._respond(error=f"Cannot flag revealed cell ({x}, {y}).",
                                 action=("flag", x, y, "error: already revealed"))
        if c in self.flags:
            self.flags.discard(c)
            return self._respond(action=("flag", x, y, "unflagged"))
        self.flags.add(c)
        return self._respond(action=("flag", x, y, "flagged"))

    def _respond(self, message: str | None = None, error: str | None = None, action=None):
        over = self.state != "playing"
        meta = {"state": self.state, "mines_remaining": self.num_mines - len(self.flags),
                "revealed_count": len(self.opened),
                "total_safe": self.width * self.height - self.num_mines, "game_over": over}
        if message:
            meta["message"] = message
        if error:
            meta["error"] = error
        if over:
            meta["early_exit"] = True
        if self.text_mode:
            text = (self.render(reveal_all=over, coords=False) + f"\n\nstate: {self.state} | mines: "
                    f"{meta['mines_remaining']} | progress: {len(self.opened)}/{meta['total_safe']}")
            if action:
                text += f"\n{action[0]}({action[1]},{action[2]}) -> {action[3]}"
            elif error:
                text += f"\nerror: {error}"
            return text, meta
        out = {"board": self.render(reveal_all=over, coords=True), **meta}
        out.pop("revealed_count")
        out.pop("total_safe")
        return out


def build_server(width: int = 9, height: int = 9, num_mines: int = 10, seed: int | None = None,
                 text_mode: bool = False, no_guess: bool = True):
    """FastMCP server with ``reveal``, ``flag`` and ``reset_game`` tools over one game."""
    from mcp.server.fastmcp import FastMCP

    game = MinesweeperGame(width, height, num_mines, seed, text_mode=text_mode, no_guess=no_guess)
    mcp = FastMCP(name="minesweeper", instructions=(
        f"Minesweeper on a {width}x{height} board with {num_mines} mines. Coordinates are (x, y) "
        "with x the column and y the row, both from 0. Symbols: '.' hidden, 'F' flagged, '_' "
        "revealed with no adjacent mines, '1'-'8' adjacent mine count, '*' mine. The first "
        "reveal is always safe. Reveal every safe cell to win."))

    def _out(r):
        if isinstance(r, tuple):            # text mode: (text, metadata)
            text, meta = r
            return {"text": text, **meta}
        return r

    @mcp.tool(description="Reveal the cell at (x, y). Cells with no adjacent mines open their "
                          "neighbours automatically. Revealing a mine ends the game.")
    def reveal(x: Annotated[int, "column, 0-based"], y: Annotated[int, "row, 0-based"]) -> dict:
        return _out(game.reveal(int(x), int(y)))

    @mcp.tool(description="Place or remove a flag on the hidden cell at (x, y).")
    def flag(x: Annotated[int, "column, 0-based"], y: Annotated[int, "row, 0-based"]) -> dict:
        return _out(game.toggle_flag(int(x), int(y)))

    @mcp.tool(description="Start a new game with the same board size and mine count.")
    def reset_game(seed: Annotated[int | None, "optional random seed"] = None) -> dict:
        game.reset(seed)
        return _out(game._respond(message="New game started."))

    mcp.game = game
    return mcp


def reward(result, metadata: dict) -> float:
    """1.0 when the last tool step reports a won game, else the fraction of safe cells opened
    times 0.5 (partial credit keeps a gradient on hard boards)."""
    for s in reversed(getattr(result, "steps", []) if result is not None else []):
        so = getattr(s, "structured_output", None)
        if so and "state" in so:
            if so["state"] == "won":
                return 1.0
            if "revealed_count" in so and so.get("total_safe"):
                return 0.5 * so["revealed_count"] / so["total_safe"]
            return 0.0
    return 0.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--width", type=int, default=9)
    ap.add_argument("--height", type=int, default=9)
    ap.add_argument("--mines", type=int, default=10)
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("--text", action="store_true", help="text board responses")
    ap.add_argument("--allow-guess", action="store_true", help="skip the no-guess layout check")
    a = ap.parse_args()
    build_server(a.width, a.height, a.mines, a.seed, a.text, not a.allow_guess).run()


if __name__ == "__main__":
    main()
