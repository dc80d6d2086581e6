"""CPU restatement of the reference path: the checker of the test suite and the CPU
baseline of the benchmark. Never imported by the product package."""
