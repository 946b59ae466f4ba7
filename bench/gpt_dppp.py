#!/usr/bin/env python
"""GPT-1B FP8, DP=2 x PP=4, 1F1B, 16 micro-batches of 4 x 2048 tokens, full
activation checkpointing per stage, on 8 GPUs of one NVSwitch node.

    torchrun --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 bench/gpt_dppp.py
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from gpt_pipeline import main  # noqa: E402

if __name__ == "__main__":
    sys.exit(main(defaults=dict(model="gpt1b", dp=2, pp=4, schedule="1f1b", micro_batches=16, micro_batch=4)))
