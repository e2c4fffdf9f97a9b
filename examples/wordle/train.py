"""Wordle: the model plays Wordle through an MCP ``guess`` tool (one server per rollout, target
word from the answer list); reward 1 for a win (the reference's examples/wordle/train.py).

    bash examples/wordle/serve.sh          # engine server(s)
    bash examples/wordle/run_train.sh      # trainer (torchrun over the training GPUs)
"""
import os
import random
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from common import base_args, mcp_server, run  # noqa: E402

from agent_factory_3_b200.envs import wordle  # noqa: E402

PROMPT = ("Let's play Wordle. Guess the hidden 5-letter English word in at most 6 attempts "
          "using the `guess` tool. Each guess returns per-letter feedback. Think about the "
          "feedback before each guess.")


def dataset(seed: int) -> list[dict]:
    words = sorted(wordle.load_words(wordle.DATA / "wordle_answers.txt"))
    random.Random(seed).shuffle(words)
    return [{"prompt": PROMPT, "target": w,
             "mcp_config": mcp_server("agent_factory_3_b200.envs.wordle", "--target", w)}
            for w in words]


if __name__ == "__main__":
    a = base_args().parse_args()
    run(a, dataset(a.seed), wordle.reward, "wordle")
