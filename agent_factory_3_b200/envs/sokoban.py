"""Sokoban as an MCP environment with text or image observations (reference environments:
mcp_tools/sokoban/server_text.py:63-380 over gym_sokoban with its deadlock detector under
mcp_tools/sokoban/deadlock_detector, and the image server mcp_tools/sokoban/server.py:19-190).

* Image mode (``build_server(..., image=True)``, ``--image``): every observation is a frame
  drawn on the CPU with numpy (16-pixel tiles, nearest-neighbour upscaled by 1.75 as in the
  reference) and sent as a JPEG image block; the tool result is [description, image(s),
  metadata], the metadata as a fenced ``metadata`` JSON text block (the reference's format,
  which the rollout executor reads as structured output).

* Levels come from our own generator: a room is carved by a random walk inside a wall border,
  targets are placed on floor cells, and the start position is made by playing the game
  backwards from the solved position (the player pulls boxes off their targets with random
  moves), so every level is solvable.  ``difficulty`` is the number of reverse pulls.
* Board text keeps the familiar symbols: ``X`` wall, ``.`` floor, ``T`` target, ``B`` box,
  ``*`` box on target, ``@`` player, ``+`` player on target; cells separated by spaces.
* Rewards per move follow the common Sokoban convention: -0.1 per step, +1 for a box pushed
  onto a target, -1 for one pushed off, +10 when every box is placed; the episode's running
  total starts at ``init_state_reward`` and the first move adds ``first_move_reward``.
* Deadlocks (checked after every push): a box on a dead square (from which no push sequence
  reaches any target, computed once by pulling from every target), a 2x2 block of walls and
  boxes with a box off target, or a box frozen on both axes by walls or other frozen boxes.
  ``early_exit`` is set on a solve or a deadlock.

    python -m agent_factory_3_b200.envs.sokoban --width 7 --height 7 --boxes 2 --seed 0
"""
from __future__ import annotations

import argparse
import random
from typing import Annotated

WALL, FLOOR = "X", "."
DIRS = {"up": (0, -1), "down": (0, 1), "left": (-1, 0), "right": (1, 0)}


class SokobanLevel:
    def __init__(self, walls: set, targets: set, boxes: set, player: tuple, w: int, h: int,
                 difficulty: int = 0):
        self.walls, self.targets, self.boxes = set(walls), set(targets), set(boxes)
        self.player, self.w, self.h, self.difficulty = player, w, h, difficulty

    def copy(self) -> "SokobanLevel":
        return SokobanLevel(self.walls, self.targets, self.boxes, self.player, self.w, self.h,
                            self.difficulty)

    def render(self) -> str:
        rows = []
        for y in range(self.h):
            cells = []
            for x in range(self.w):
                c = (x, y)
                if c in self.walls:
                    cells.append(WALL)
                elif c == self.player:
                    cells.append("+" if c in self.targets else "@")
                elif c in self.boxes:
                    cells.append("*" if c in self.targets else "B")
                else:
                    cells.append("T" if c in self.targets else FLOOR)
            rows.append(" ".join(cells))
        return "\n".join(rows) + "\n"

    def solved(self) -> bool:
        return self.boxes == self.targets


def generate_level(w: int = 7, h: int = 7, num_boxes: int = 2, seed: int | None = None,
                   walk_steps: int | None = None, pulls: int | None = None,
                   max_tries: int = 200) -> SokobanLevel:
    """Random solvable level (carve, place targets, then pull boxes backwards)."""
    rng = random.Random(seed)
    if w < 5 or h < 5:
        raise ValueError("room must be at least 5x5")
    interior = [(x, y) for y in range(1, h - 1) for x in range(1, w - 1)]
    for _ in range(max_tries):
        floor = set()
        cur = rng.choice(interior)
        for _ in range(walk_steps or (w * h)):
            floor.add(cur)
            dx, dy = rng.choice(list(DIRS.values()))
            nxt = (cur[0] + dx, cur[1] + dy)
            if 1 <= nxt[0] < w - 1 and 1 <= nxt[1] < h - 1:
                cur = nxt
        if len(floor) < num_boxes + 3:
            continue
        walls = {(x, y) for y in range(h) for x in range(w)} - floor
        cells = sorted(floor)
        targets = set(rng.sample(cells, num_boxes))
        boxes = set(targets)
        player = rng.choice([c for c in cells if c not in boxes])
        n_pulls = 0
        for _ in range(pulls or 40 * num_boxes):
            dx, dy = rng.choice(list(DIRS.values()))
            step = (player[0] + dx, player[1] + dy)
            if step in walls or step in boxes:
                continue
            behind = (player[0] - dx, player[1] - dy)   # box behind the player gets pulled
            if behind in boxes and rng.random() < 0.8:
                boxes.discard(behind)
                boxes.add(player)
                n_pulls += 1
            player = step
        if boxes != targets and n_pulls > 0:
            return SokobanLevel(walls, targets, boxes, player, w, h, difficulty=n_pulls)
    raise RuntimeError("could not generate a level; try a larger room or fewer boxes")


def live_squares(level: SokobanLevel) -> set:
    """Squares from which a box can still reach some target: pull boxes from every target."""
    live = set(level.targets)
    stack = list(level.targets)
    while stack:
        c = stack.pop()
        for dx, dy in DIRS.values():
            prev = (c[0] + dx, c[1] + dy)          # box came from here ...
            stand = (c[0] + 2 * dx, c[1] + 2 * dy)  # ... pushed by a player standing here
            if prev not in level.walls and stand not in level.walls and prev not in live:
                live.add(prev)
                stack.append(prev)
    return live


def find_deadlocks(level: SokobanLevel, live: set | None = None) -> list[str]:
    live = live if live is not None else live_squares(level)
    reasons = []
    for b in sorted(level.boxes):
        if b not in level.targets and b not in live:
            reasons.append(f"box at {b} is on a dead square (cannot reach any target)")
    blocked = level.walls | level.boxes
    for x in range(level.w - 1):
        for y in range(level.h - 1):
            quad = [(x, y), (x + 1, y), (x, y + 1), (x + 1, y + 1)]
            if all(c in blocked for c in quad) and any(
                    c in level.boxes and c not in level.targets for c in quad):
                reasons.append(f"2x2 block of walls/boxes at {(x, y)} with a box off target")
    frozen: set = set()
    changed = True
    while changed:                       # boxes that can move on neither axis
        changed = False
        for b in level.boxes:
            if b in frozen:
                continue
            stuck = []
            for axis in ((1, 0), (0, 1)):
                a = (b[0] - axis[0], b[1] - axis[1])
                c = (b[0] + axis[0], b[1] + axis[1])
                stuck.append(a in level.walls or c in level.walls or a in frozen or c in frozen)
            if all(stuck):
                frozen.add(b)
                changed = True
    for b in sorted(frozen - level.targets):
        reasons.append(f"box at {b} is frozen off target")
    return reasons


class SokobanGame:
    def __init__(self, width: int = 7, height: int = 7, num_boxes: int = 2, seed: int | None = None,
                 init_state_reward: float = 3.0, first_move_reward: float = 3.0,
                 max_moves_per_call: int = 5):
        self.cfg = dict(w=width, h=height, num_boxes=num_boxes)
        self.init_state_reward = init_state_reward
        self.first_move_reward = first_move_reward
        self.max_moves_per_call = max_moves_per_call
        self.reset(seed)

    def reset(self, seed: int | None = None) -> None:
        self.seed = seed
        self.level = generate_level(seed=seed, **self.cfg)
        self.live = live_squares(self.level)
        self.steps = 0
        self.history: list[str] = []
        self.total_reward = self.init_state_reward
        self.done = False

    def step(self, direction: str) -> tuple[float, bool, bool]:
        """One move: (reward, moved a box, solved)."""
        dx, dy = DIRS[direction]
        lv = self.level
        nxt = (lv.player[0] + dx, lv.player[1] + dy)
        reward, pushed = -0.1, False
        if nxt in lv.walls:
            pass
        elif nxt in lv.boxes:
            beyond = (nxt[0] + dx, nxt[1] + dy)
            if beyond not in lv.walls and beyond not in lv.boxes:
                lv.boxes.discard(nxt)
                lv.boxes.add(beyond)
                reward += (beyond in lv.targets) - (nxt in lv.targets)
                lv.player, pushed = nxt, True
        else:
            lv.player = nxt
        solved = lv.solved()
        if solved:
            reward += 10.0
            self.done = True
        if self.steps == 0:
            reward += self.first_move_reward
        self.steps += 1
        self.history.append(direction)
        self.total_reward += reward
        return reward, pushed, solved

    def meta(self, **extra) -> dict:
        return {"seed": self.seed, "step_count": self.steps, "accumulated_reward": self.total_reward,
                "move_history": list(self.history), "difficulty": self.level.difficulty, **extra}


# ------------------------------------------------------------------ image observations
TILE = 16
UPSCALE = 1.75
_COLORS = {"wall": (96, 64, 48), "floor": (24, 24, 24), "target": (200, 40, 40),
           "box": (220, 170, 40), "box_on_target": (60, 190, 60), "player": (70, 130, 230)}


def _tile(kind: str, on_target: bool):
    import numpy as np
    t = np.empty((TILE, TILE, 3), np.uint8)
    t[:] = _COLORS["wall" if kind == "wall" else "floor"]
    if kind == "wall":
        t[::4, :] = (72, 48, 36)                       # brick courses
        return t
    if on_target:                                      # red outline of the target square
        t[2:14, 2:4] = t[2:14, 12:14] = _COLORS["target"]
        t[2:4, 2:14] = t[12:14, 2:14] = _COLORS["target"]
    if kind == "box":
        t[3:13, 3:13] = _COLORS["box_on_target" if on_target else "box"]
        t[7:9, 3:13] = t[3:13, 7:9] = (90, 60, 20)     # box cross-beams
    elif kind == "player":
        yy, xx = np.mgrid[0:TILE, 0:TILE]
        t[(yy - 7.5) ** 2 + (xx - 7.5) ** 2 <= 20] = _COLORS["player"]
    return t


def render_frame(level: SokobanLevel, upscale: float = UPSCALE):
    """RGB uint8 [H, W, 3] frame of the board (numpy tiles, nearest-neighbour upscale)."""
    import numpy as np
    img = np.empty((level.h * TILE, level.w * TILE, 3), np.uint8)
    for y in range(level.h):
        for x in range(level.w):
            c = (x, y)
            on_t = c in level.targets
            kind = ("wall" if c in level.walls else "player" if c == level.player
                    else "box" if c in level.boxes else "floor")
            img[y * TILE:(y + 1) * TILE, x * TILE:(x + 1) * TILE] = _tile(kind, on_t)
    if upscale != 1.0:
        H, W = int(img.shape[0] * upscale), int(img.shape[1] * upscale)
        ys = (np.arange(H) / upscale).astype(int)
        xs = (np.arange(W) / upscale).astype(int)
        img = img[ys][:, xs]
    return img


def frame_jpeg(level: SokobanLevel, quality: int = 90) -> bytes:
    import io

    from PIL import Image as PILImage
    buf = io.BytesIO()
    PILImage.fromarray(render_frame(level)).save(buf, format="JPEG", quality=quality)
    return buf.getvalue()


def metadata_block(meta: dict) -> str:
    import json
    return f"```metadata\n{json.dumps(meta, indent=2)}\n```"


def build_server(width: int = 7, height: int = 7, num_boxes: int = 2, seed: int | None = None,
                 image: bool = False):
    """FastMCP server with ``get_init_state`` and ``move_sequence`` over one game (text board,
    or JPEG frames with ``image``)."""
    from mcp.server.fastmcp import FastMCP
    if image:
        return _build_image_server(width, height, num_boxes, seed)

    game = SokobanGame(width, height, num_boxes, seed)
    mcp = FastMCP(name="sokoban", instructions=(
        "Sokoban: push every box (B) onto a target (T). You are @ (+ when on a target); X is a "
        "wall, . is floor, * is a box on a target. You can push one box at a time and never "
        "pull. Call get_init_state to see the board, then move_sequence with up to "
        f"{game.max_moves_per_call} directions (up, down, left, right) per call."))

    @mcp.tool(description="Return the current board (call once at the start).")
    def get_init_state() -> dict:
        return {"text": game.level.render(), **game.meta(early_exit=False, is_passed=False,
                                                         is_deadlock=False)}

    @mcp.tool(description="Make up to 5 moves in order; stops early on a solve or a deadlock.")
    def move_sequence(directions: Annotated[list[str], "moves, e.g. [\"up\", \"left\"] (max 5)"]) -> dict:
        if len(directions) > game.max_moves_per_call:
            return {"error": f"Maximum {game.max_moves_per_call} moves allowed, got {len(directions)}.",
                    **game.meta(early_exit=False, is_passed=False, is_deadlock=False)}
        if game.done:
            return {"error": "Game already completed.", **game.meta(early_exit=True, is_passed=True,
                                                                     is_deadlock=False)}
        lines, passed, deadlock = [], False, []
        for d in directions:
            d = str(d).lower()
            if d not in DIRS:
                lines.append(f"Error: invalid direction '{d}'. Valid directions: {sorted(DIRS)}")
                break
            _, pushed, solved = game.step(d)
            lines.append(f"Step {game.steps}, Move: {d}\n{game.level.render()}")
            if pushed:
                deadlock = find_deadlocks(game.level, game.live)
            if deadlock:
                lines.append("Deadlock detected!\n" + "\n".join(f"  - {r}" for r in deadlock))
                break
            if solved:
                lines.append("Congratulations! You solved the puzzle!")
                passed = True
                break
        if not passed and not deadlock:
            lines.append("Not yet solved, please continue.")
        return {"text": "\n".join(lines), **game.meta(early_exit=passed or bool(deadlock),
                                                      is_passed=passed, is_deadlock=bool(deadlock))}

    mcp.game = game
    return mcp


def _build_image_server(width: int, height: int, num_boxes: int, seed: int | None):
    from mcp.server.fastmcp import FastMCP, Image

    game = SokobanGame(width, height, num_boxes, seed)
    mcp = FastMCP(name="sokoban-image", instructions=(
        "Sokoban: push every yellow box onto a red-outlined target (a box on a target turns "
        "green). You are the blue circle; brown cells are walls. Call get_init_state to see the "
        f"board, then move_sequence with up to {game.max_moves_per_call} directions "
        "(up, down, left, right) per call."))

    @mcp.tool(description="Return the current board as an image (call once at the start).")
    def get_init_state() -> list:
        meta = game.meta(early_exit=False, is_passed=False, is_deadlock=False)
        return ["Sokoban game initialized. Ready to play! Use move_sequence to make moves.",
                Image(data=frame_jpeg(game.level), format="jpeg"), metadata_block(meta)]

    @mcp.tool(description="Make up to 5 moves in order; an image after each move; stops early "
                          "on a solve or a deadlock.")
    def move_sequence(directions: Annotated[list[str], "moves, e.g. [\"up\", \"left\"] (max 5)"]) -> list:
        if len(directions) > game.max_moves_per_call:
            return [f"Error: Maximum {game.max_moves_per_call} moves allowed, got {len(directions)}.",
                    metadata_block(game.meta(early_exit=False, is_passed=False, is_deadlock=False))]
        if game.done:
            return ["Error: Game already completed.",
                    metadata_block(game.meta(early_exit=True, is_passed=True, is_deadlock=False))]
        out: list = []
        passed, deadlock = False, []
        for d in directions:
            d = str(d).lower()
            if d not in DIRS:
                out.append(f"Error: invalid direction '{d}'. Valid directions: {sorted(DIRS)}")
                break
            _, pushed, solved = game.step(d)
            if pushed:
                deadlock = find_deadlocks(game.level, game.live)
            if solved:
                out.append("Congratulations! You solved the puzzle!")
                passed = True
                break
            out += [f"Step {game.steps}, Move: {d}", Image(data=frame_jpeg(game.level), format="jpeg")]
            if deadlock:
                out.append("Deadlock detected!\n" + "\n".join(f"  - {r}" for r in deadlock))
                break
        out.append(metadata_block(game.meta(early_exit=passed or bool(deadlock), is_passed=passed,
                                            is_deadlock=bool(deadlock))))
        return out

    mcp.game = game
    return mcp


def reward(result, metadata: dict) -> float:
    """1.0 for a solved puzzle, else 0.0."""
    for s in reversed(getattr(result, "steps", []) if result is not None else []):
        so = getattr(s, "structured_output", None)
        if so and "is_passed" in so:
            return 1.0 if so["is_passed"] else 0.0
    return 0.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--width", type=int, default=7)
    ap.add_argument("--height", type=int, default=7)
    ap.add_argument("--boxes", type=int, default=2)
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("--image", action="store_true", help="JPEG frame observations")
    a = ap.parse_args()
    build_server(a.width, a.height, a.boxes, a.seed, image=a.image).run()


if __name__ == "__main__":
    main()
