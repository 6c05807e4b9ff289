"""CPU oracle of the ALUT path - test infrastructure only (parity checker, CPU baseline)."""
