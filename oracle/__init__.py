"""CPU oracle of the reference's FP32 arithmetic -- test infrastructure only."""
