"""B200-native (sm_100a) quantized-weight matrix path of Siphon."""
