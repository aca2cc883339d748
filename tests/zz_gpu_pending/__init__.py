"""GPU tests written without GPU time, collected after every other test until a B200 run has confirmed them."""
