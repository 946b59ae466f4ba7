#!/usr/bin/env python
"""GPT-3-style 6.7B FP8 (32 layers, d 4096, 32 heads, d_ff 16384, vocab 50304,
seq 2048), GPipe over 8 stages, 32 micro-batches of 2 sequences, full activation
checkpointing per stage; reports the measured bubble next to (S-1)/(M+S-1).

    torchrun --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 bench/gpt67b_gpipe.py
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from gpt_pipeline import main  # noqa: E402

if __name__ == "__main__":
    sys.exit(main(defaults=dict(model="gpt6.7b", dp=1, pp=8, schedule="gpipe", micro_batches=32, micro_batch=2)))
