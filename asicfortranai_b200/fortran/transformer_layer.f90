! Drop-in replacement of module transformer_layer (transformer_layer.f90) over libq35.so.
! Same public names.  TransformerLayer keeps the reference's components -- the host arrays
! a caller fills (weights in the reference's W_Q(K/2,N) layout, per-column scales, norms),
! the RoPE table, the KV-cache arrays and cache_pos -- and gains:
!   handle       the layer on the GPU (a one-layer libq35 model), made by the first
!                apply_transformer_layer from the host arrays and reused afterwards; the
!                live KV cache is the device one (the host k_cache/v_cache arrays are
!                allocated and zeroed as the reference does, and not written);
!   *_offsets    per-column offsets: when wq_offsets is allocated the layer's matrices are
!                3.5-bit codes (matmul_3p5bit_dynamic.f90), else INT4 (matmul_int4_groq.f90);
!   max_seq_len  the KV-cache length, from init_kv_cache (2048 when never called).
! Sizes come from the arrays (hidden = 2*size(wq,1), query heads = size(wq,2)/HEAD_DIM,
! KV heads = size(wk,2)/HEAD_DIM, FFN = size(w_gate,2)), so configurations other than the
! 70B constants work too.  After changing a layer's host weights call sync_layer_weights
! (or release_layer) so the next application uploads them again.  Every procedure takes
! an optional stat=; without it a failure stops with libq35's message (q35_status).
! Compile after q35_status.f90 and q35_model_api.f90.
module transformer_layer
    use iso_c_binding, only: c_int, c_int32_t, c_float, c_ptr, c_null_ptr, c_associated, c_loc
    use iso_fortran_env, only: int8, int32, real32
    use q35_status, only: q35_check
    use q35_model_api
    implicit none
    private
    public :: TransformerLayer, apply_transformer_layer, init_rope_freqs
    public :: init_kv_cache, reset_kv_cache, rms_norm
    public :: HIDDEN_DIM, INTERMEDIATE_DIM, NUM_HEADS, NUM_KV_HEADS, HEAD_DIM
    public :: sync_layer_weights, release_layer, upload_layer, layer_config, layer_weights_view
    public :: layer_weights_loaded

    ! LLaMA 70B configuration (transformer_layer.f90:21-27)
    integer(int32), parameter :: HIDDEN_DIM = 8192
    integer(int32), parameter :: INTERMEDIATE_DIM = 28672
    integer(int32), parameter :: NUM_HEADS = 64
    integer(int32), parameter :: NUM_KV_HEADS = 8
    integer(int32), parameter :: HEAD_DIM = 128
    real(real32), parameter :: RMS_NORM_EPS = 1.0e-5

    ! transformer_layer.f90:30-60, plus the device handle and the 3.5-bit offsets
    type :: TransformerLayer
        integer(int8), allocatable :: wq(:,:), wk(:,:), wv(:,:), wo(:,:)
        real(real32), allocatable :: wq_scales(:), wk_scales(:), wv_scales(:), wo_scales(:)
        integer(int8), allocatable :: w_gate(:,:), w_up(:,:), w_down(:,:)
        real(real32), allocatable :: w_gate_scales(:), w_up_scales(:), w_down_scales(:)
        real(real32), allocatable :: attn_norm(:), ffn_norm(:)
        real(real32), allocatable :: rope_freqs(:,:)
        real(real32), allocatable :: k_cache(:,:,:), v_cache(:,:,:)
        integer(int32) :: cache_pos = 0
        real(real32), allocatable :: wq_offsets(:), wk_offsets(:), wv_offsets(:), wo_offsets(:)
        real(real32), allocatable :: w_gate_offsets(:), w_up_offsets(:), w_down_offsets(:)
        integer(int32) :: max_seq_len = 0
        type(c_ptr) :: handle = c_null_ptr
    end type TransformerLayer

contains

    ! the device configuration of a layer (one layer; vocabulary 1: a layer alone has no
    ! embedding or LM head to speak of)
    function layer_config(layer, n_layers, vocab, max_seq) result(cfg)
        type(TransformerLayer), intent(in) :: layer
        integer(int32), intent(in) :: n_layers, vocab, max_seq
        type(q35_model_config_t) :: cfg
        cfg%n_layers = n_layers
        cfg%hidden = 2 * size(layer%wq, 1)
        cfg%n_heads = size(layer%wq, 2) / HEAD_DIM
        cfg%n_kv_heads = size(layer%wk, 2) / HEAD_DIM
        cfg%head_dim = HEAD_DIM
        cfg%ffn = size(layer%w_gate, 2)
        cfg%vocab = vocab
        cfg%max_seq = max_seq
        cfg%rms_eps = RMS_NORM_EPS
        cfg%rope_theta = 10000.0
        cfg%rope_mode = 0            ! the position within the call (transformer_layer.f90:193-196)
        cfg%wformat = Q35_FMT_INT4
        if (allocated(layer%wq_offsets)) cfg%wformat = Q35_FMT_3P5BIT
        cfg%max_batch = 1
    end function layer_config

    ! the addresses of a layer's host arrays as libq35 reads them (the layer must be a
    ! target and its weight arrays allocated)
    function layer_weights_view(layer) result(lw)
        type(TransformerLayer), intent(in), target :: layer
        type(q35_layer_weights_t) :: lw
        lw%wq = c_loc(layer%wq)
        lw%wk = c_loc(layer%wk)
        lw%wv = c_loc(layer%wv)
        lw%wo = c_loc(layer%wo)
        lw%wg = c_loc(layer%w_gate)
        lw%wu = c_loc(layer%w_up)
        lw%wd = c_loc(layer%w_down)
        lw%sq = c_loc(layer%wq_scales)
        lw%sk = c_loc(layer%wk_scales)
        lw%sv = c_loc(layer%wv_scales)
        lw%so = c_loc(layer%wo_scales)
        lw%sg = c_loc(layer%w_gate_scales)
        lw%su = c_loc(layer%w_up_scales)
        lw%sd = c_loc(layer%w_down_scales)
        if (allocated(layer%wq_offsets)) then
            lw%oq = c_loc(layer%wq_offsets)
            lw%ok = c_loc(layer%wk_offsets)
            lw%ov = c_loc(layer%wv_offsets)
            lw%oo = c_loc(layer%wo_offsets)
            lw%og = c_loc(layer%w_gate_offsets)
            lw%ou = c_loc(layer%w_up_offsets)
            lw%od = c_loc(layer%w_down_offsets)
        end if
        if (allocated(layer%attn_norm)) lw%attn_norm = c_loc(layer%attn_norm)
        if (allocated(layer%ffn_norm)) lw%ffn_norm = c_loc(layer%ffn_norm)
    end function layer_weights_view

    ! every matrix and its scales allocated (what the device copy is made from)
    logical function layer_weights_loaded(layer)
        type(TransformerLayer), intent(in) :: layer
        layer_weights_loaded = allocated(layer%wq) .and. allocated(layer%wk) .and. allocated(layer%wv) .and. &
                          allocated(layer%wo) .and. allocated(layer%w_gate) .and. allocated(layer%w_up) .and. &
                          allocated(layer%w_down) .and. allocated(layer%wq_scales) .and. &
                          allocated(layer%wk_scales) .and. allocated(layer%wv_scales) .and. &
                          allocated(layer%wo_scales) .and. allocated(layer%w_gate_scales) .and. &
                          allocated(layer%w_up_scales) .and. allocated(layer%w_down_scales)
    end function layer_weights_loaded

    ! upload the layer to the GPU when it has no device copy yet
    subroutine upload_layer(layer, stat)
        type(TransformerLayer), intent(inout), target :: layer
        integer, intent(out), optional :: stat
        type(q35_model_config_t) :: cfg
        type(q35_layer_weights_t) :: lw
        type(c_ptr) :: ctx
        integer :: st
        if (present(stat)) stat = 0
        if (c_associated(layer%handle)) return
        if (.not. layer_weights_loaded(layer)) then
            if (present(stat)) then
                stat = 1
                return
            end if
            error stop "apply_transformer_layer: the layer's weight arrays are not allocated"
        end if
        ctx = q35_fortran_context(st)
        if (st /= 0) then
            call q35_check(int(st, c_int), "apply_transformer_layer", stat)
            return
        end if
        if (layer%max_seq_len <= 0) layer%max_seq_len = 2048
        cfg = layer_config(layer, 1, 1, layer%max_seq_len)
        st = q35_model_create(ctx, cfg, layer%handle)
        if (st == 0) then
            lw = layer_weights_view(layer)
            st = q35_model_set_layer(layer%handle, 0_c_int32_t, lw)
        end if
        call q35_check(int(st, c_int), "apply_transformer_layer (upload)", stat)
    end subroutine upload_layer

    ! transformer_layer.f90:96-118: the RoPE angle table (host), as the reference builds it;
    ! the GPU builds the same table with the same formula for its kernels
    subroutine init_rope_freqs(layer, max_seq_len)
        type(TransformerLayer), intent(inout) :: layer
        integer(int32), intent(in) :: max_seq_len
        integer(int32) :: pos, d
        real(real32) :: theta, freq_base
        if (.not. allocated(layer%rope_freqs)) allocate(layer%rope_freqs(max_seq_len, HEAD_DIM/2))
        freq_base = 10000.0
        do d = 1, HEAD_DIM/2
            theta = freq_base ** (-2.0 * real(d-1, real32) / real(HEAD_DIM, real32))
            do pos = 1, max_seq_len
                layer%rope_freqs(pos, d) = real(pos-1, real32) * theta
            end do
        end do
        if (layer%max_seq_len <= 0) layer%max_seq_len = max_seq_len
    end subroutine init_rope_freqs

    ! transformer_layer.f90:124-140: the cache length and a cleared cache
    subroutine init_kv_cache(layer, max_seq_len, stat)
        type(TransformerLayer), intent(inout) :: layer
        integer(int32), intent(in) :: max_seq_len
        integer, intent(out), optional :: stat
        if (present(stat)) stat = 0
        if (.not. allocated(layer%k_cache)) allocate(layer%k_cache(max_seq_len, NUM_KV_HEADS, HEAD_DIM))
        if (.not. allocated(layer%v_cache)) allocate(layer%v_cache(max_seq_len, NUM_KV_HEADS, HEAD_DIM))
        layer%k_cache = 0.0
        layer%v_cache = 0.0
        layer%cache_pos = 0
        if (c_associated(layer%handle) .and. layer%max_seq_len /= max_seq_len) then
            call release_layer(layer)              ! the device cache is re-made at the new length
        else if (c_associated(layer%handle)) then
            call q35_check(q35_model_reset(layer%handle), "init_kv_cache", stat)
        end if
        layer%max_seq_len = max_seq_len
    end subroutine init_kv_cache

    ! transformer_layer.f90:145-150
    subroutine reset_kv_cache(layer, stat)
        type(TransformerLayer), intent(inout) :: layer
        integer, intent(out), optional :: stat
        if (present(stat)) stat = 0
        layer%cache_pos = 0
        if (allocated(layer%k_cache)) layer%k_cache = 0.0
        if (allocated(layer%v_cache)) layer%v_cache = 0.0
        if (c_associated(layer%handle)) call q35_check(q35_model_reset(layer%handle), "reset_kv_cache", stat)
    end subroutine reset_kv_cache

    ! transformer_layer.f90:155-178, on the GPU (rmsnorm_kernel)
    subroutine rms_norm(x, weight, output, seq_len, dim, stat)
        integer(int32), intent(in), value :: seq_len, dim
        real(real32), intent(in) :: x(seq_len, dim)
        real(real32), intent(in) :: weight(dim)
        real(real32), intent(out) :: output(seq_len, dim)
        integer, intent(out), optional :: stat
        call q35_check(q35_rms_norm(x, weight, output, seq_len, dim), "rms_norm", stat)
    end subroutine rms_norm

    ! transformer_layer.f90:527-565: x -> x + attention(RMSNorm(x)) -> + SwiGLU FFN(RMSNorm(.))
    ! on the GPU, with the layer's KV cache advanced by seq_len positions
    subroutine apply_transformer_layer(layer, x, output, seq_len, stat)
        type(TransformerLayer), intent(inout), target :: layer
        integer(int32), intent(in), value :: seq_len
        real(real32), intent(in) :: x(seq_len, *)
        real(real32), intent(out) :: output(seq_len, *)
        integer, intent(out), optional :: stat
        integer :: st
        call upload_layer(layer, st)
        if (st /= 0) then
            call q35_check(int(st, c_int), "apply_transformer_layer", stat)
            return
        end if
        st = q35_model_layer_forward(layer%handle, 0_c_int32_t, 0_c_int32_t, x, seq_len, output, 1_c_int32_t)
        if (st == 0) layer%cache_pos = layer%cache_pos + seq_len
        call q35_check(int(st, c_int), "apply_transformer_layer", stat)
    end subroutine apply_transformer_layer

    ! re-upload the layer's host weights and norms to its device copy (after editing them)
    subroutine sync_layer_weights(layer, stat)
        type(TransformerLayer), intent(inout), target :: layer
        integer, intent(out), optional :: stat
        type(q35_layer_weights_t) :: lw
        if (present(stat)) stat = 0
        if (.not. c_associated(layer%handle)) return
        lw = layer_weights_view(layer)
        call q35_check(q35_model_set_layer(layer%handle, 0_c_int32_t, lw), "sync_layer_weights", stat)
    end subroutine sync_layer_weights

    ! drop the layer's device copy (the next application uploads it again)
    subroutine release_layer(layer)
        type(TransformerLayer), intent(inout) :: layer
        integer(c_int) :: st
        if (c_associated(layer%handle)) then
            st = q35_model_destroy(layer%handle)
            layer%handle = c_null_ptr
        end if
    end subroutine release_layer

end module transformer_layer
