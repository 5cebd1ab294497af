"""B200 token loop for the Llama-style models of tmc/ane-training-experiments.

Sub-packages mirror the reference's Go packages on the path: `stories` (decoder, weights,
tokenizer, file formats) and `storiesane` (full-window evaluation and windowed decode) over the
CUDA C ABI in `_abi`; `shard` partitions sequences across ranks.
"""
