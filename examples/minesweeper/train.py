"""Minesweeper: the model clears a no-guess 9x9 board with 10 mines through MCP ``reveal`` /
``flag`` tools (text board responses); reward 1 for a cleared board (the reference's
examples/minesweeper/train.py).

    bash examples/minesweeper/serve.sh
    bash examples/minesweeper/run_train.sh
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from common import base_args, mcp_server, run  # noqa: E402

from agent_factory_3_b200.envs import minesweeper  # noqa: E402

PROMPT = ("Play Minesweeper on a 9x9 board with 10 mines. Use `reveal` to open a cell and `flag` "
          "to mark a mine; the board is shown after every move. Clear every safe cell to win.")


def dataset(n: int, seed: int) -> list[dict]:
    return [{"prompt": PROMPT, "board_seed": seed * 100003 + i,
             "mcp_config": mcp_server("agent_factory_3_b200.envs.minesweeper", "--text",
                                      "--seed", str(seed * 100003 + i))}
            for i in range(n)]


if __name__ == "__main__":
    ap = base_args()
    ap.add_argument("--boards", type=int, default=20000)
    a = ap.parse_args()
    run(a, dataset(a.boards, a.seed), minesweeper.reward, "minesweeper")
