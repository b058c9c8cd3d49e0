"""Evaluation of candidate kernels against the B200 contract: the contract header
(kp_contract.cuh), the worker that compiles a candidate for sm_100a and runs it
through the parity and benchmark harness, the sandbox that runs the worker in a child
process, and the prompt text of the contract."""
