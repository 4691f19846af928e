"""Experiment drivers (run_single.sh, run_experiment_matrix.sh, run_node.sh,
capture_serial_prefill.sh), reports and audits over the timing JSON files,
pipeline plots, the A2F/F2A transfer benchmark, and the reference-arm runner
used by bench.py."""
