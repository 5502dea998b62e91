//! The activation-quantisation contract of the IQ2 matmul (reference src/activation_quant.rs:7-44):
//! the same two types, so that callers written against the reference compile unchanged.

/// How the activations enter the matmul.
#[derive(Clone, Copy, Debug, Default, Eq, PartialEq)]
pub enum ActivationQuantMode {
    /// Float activations (the default).
    #[default]
    Off,
    /// Every x row quantised to int8 (scale 127 / max|x|) before the matmul.
    W8A8,
    /// Not implemented by the reference either: strict callers get an error, others the float path.
    W4A8,
}

/// The mode, and whether an unsupported mode is an error (`strict`) or falls back to `Off`.
#[derive(Clone, Debug, Default, Eq, PartialEq)]
pub struct ActivationQuantConfig {
    pub mode: ActivationQuantMode,
    pub strict: bool,
}

impl ActivationQuantConfig {
    /// True unless the mode is `Off`.
    pub fn is_enabled(&self) -> bool {
        self.mode != ActivationQuantMode::Off
    }
}
