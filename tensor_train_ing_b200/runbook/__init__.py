"""Operational tools for running experiments with this framework on B200 boxes (the reference's
``scripts/`` layer, tnlm scripts/README.md): a day-one canary that gates a new box on numerics and
throughput, a trainer smoke (train, resume, replay check, evaluation), steady-state throughput and
regression checks over run directories, a scaling-law grid (plan, run, Chinchilla fit), run
audits (epoch over-read, descriptor search, stability trace) and experiment-result tools (learning
rate optimum fits, n-gram contamination, evaluated checkpoints, a weight-free results mirror).  Each module is runnable with
``python -m tensor_train_ing_b200.runbook.<tool>``.
"""
