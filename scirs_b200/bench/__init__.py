"""Benchmark harnesses for the configurations beyond the headline GPT run:
collective sweeps (`allreduce`), attention sweeps (`attention`)."""
