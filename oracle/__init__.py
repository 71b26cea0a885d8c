"""CPU oracle of the reference arithmetic -- TEST INFRASTRUCTURE ONLY (see oracle/tgo.h)."""
