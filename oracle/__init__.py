"""Oracle (test infrastructure only): the reference engine's CPU path restated in C."""
