"""Oracle package: the CPU checker for torch_ans_b200 (test infrastructure only; see oracle.py)."""
