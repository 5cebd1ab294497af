"""Command-line mirrors of the reference's cmd/ programs on the CUDA token loop."""
