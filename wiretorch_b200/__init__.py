"""B200-native engine for wiretorch's conductance-based LIF simulation step."""
