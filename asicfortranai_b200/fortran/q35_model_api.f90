! ISO_C_BINDING view of libq35's model, context and resident-weight entry points
! (include/q35.h), shared by the drop-in modules transformer_layer, llama_model,
! transformer_layer_gpu, llama_model_gpu and matmul_cublas.  The two C structs are
! mirrored field for field (q35_model_config, q35_layer_weights).
! Compile after q35_status.f90: gfortran -c q35_status.f90 q35_model_api.f90
module q35_model_api
    use iso_c_binding, only: c_int, c_int8_t, c_int32_t, c_float, c_ptr, c_null_ptr, c_associated
    use q35_status, only: q35_check
    implicit none
    private
    public :: q35_model_config_t, q35_layer_weights_t
    public :: q35_ctx_create, q35_ctx_destroy, q35_model_create, q35_model_destroy
    public :: q35_model_set_layer, q35_model_set_embeddings, q35_model_forward
    public :: q35_model_layer_forward, q35_model_reset, q35_rms_norm
    public :: q35_weights_upload, q35_weights_free, q35_matmul_cached, q35_matmul_int4_fused
    public :: q35_fortran_context, q35_fortran_context_release
    public :: Q35_FMT_3P5BIT, Q35_FMT_INT4

    integer(c_int), parameter :: Q35_FMT_3P5BIT = 0, Q35_FMT_INT4 = 1

    ! q35_model_config (include/q35.h)
    type, bind(C) :: q35_model_config_t
        integer(c_int32_t) :: n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, max_seq
        real(c_float) :: rms_eps, rope_theta
        integer(c_int32_t) :: rope_mode, wformat, max_batch
    end type q35_model_config_t

    ! q35_layer_weights (include/q35.h): the TransformerLayer matrices in the reference layout
    type, bind(C) :: q35_layer_weights_t
        type(c_ptr) :: wq = c_null_ptr, wk = c_null_ptr, wv = c_null_ptr, wo = c_null_ptr
        type(c_ptr) :: wg = c_null_ptr, wu = c_null_ptr, wd = c_null_ptr
        type(c_ptr) :: sq = c_null_ptr, sk = c_null_ptr, sv = c_null_ptr, so = c_null_ptr
        type(c_ptr) :: sg = c_null_ptr, su = c_null_ptr, sd = c_null_ptr
        type(c_ptr) :: oq = c_null_ptr, ok = c_null_ptr, ov = c_null_ptr, oo = c_null_ptr
        type(c_ptr) :: og = c_null_ptr, ou = c_null_ptr, od = c_null_ptr
        type(c_ptr) :: attn_norm = c_null_ptr, ffn_norm = c_null_ptr
    end type q35_layer_weights_t

    ! the context (device 0, a stream of its own) the Fortran model modules build on
    type(c_ptr), save :: fortran_ctx = c_null_ptr

    interface
        integer(c_int) function q35_ctx_create(device, stream, out) bind(C, name="q35_ctx_create")
            import :: c_int, c_ptr
            integer(c_int), intent(in), value :: device
            type(c_ptr), intent(in), value :: stream
            type(c_ptr), intent(out) :: out
        end function q35_ctx_create

        integer(c_int) function q35_ctx_destroy(ctx) bind(C, name="q35_ctx_destroy")
            import :: c_int, c_ptr
            type(c_ptr), intent(in), value :: ctx
        end function q35_ctx_destroy

        integer(c_int) function q35_model_create(ctx, cfg, out) bind(C, name="q35_model_create")
            import :: c_int, c_ptr, q35_model_config_t
            type(c_ptr), intent(in), value :: ctx
            type(q35_model_config_t), intent(in) :: cfg
            type(c_ptr), intent(out) :: out
        end function q35_model_create

        integer(c_int) function q35_model_destroy(m) bind(C, name="q35_model_destroy")
            import :: c_int, c_ptr
            type(c_ptr), intent(in), value :: m
        end function q35_model_destroy

        integer(c_int) function q35_model_set_layer(m, layer, w) bind(C, name="q35_model_set_layer")
            import :: c_int, c_int32_t, c_ptr, q35_layer_weights_t
            type(c_ptr), intent(in), value :: m
            integer(c_int32_t), intent(in), value :: layer
            type(q35_layer_weights_t), intent(in) :: w
        end function q35_model_set_layer

        integer(c_int) function q35_model_set_embeddings(m, embed, final_norm, lm_head) &
                bind(C, name="q35_model_set_embeddings")
            import :: c_int, c_float, c_ptr
            type(c_ptr), intent(in), value :: m
            real(c_float), intent(in) :: embed(*), final_norm(*), lm_head(*)
        end function q35_model_set_embeddings

        integer(c_int) function q35_model_forward(m, seq, ids, S, logits) bind(C, name="q35_model_forward")
            import :: c_int, c_int32_t, c_ptr
            type(c_ptr), intent(in), value :: m
            integer(c_int32_t), intent(in), value :: seq, S
            integer(c_int32_t), intent(in) :: ids(*)
            type(c_ptr), intent(in), value :: logits
        end function q35_model_forward

        integer(c_int) function q35_model_layer_forward(m, layer, seq, x, S, out, advance) &
                bind(C, name="q35_model_layer_forward")
            import :: c_int, c_int32_t, c_float, c_ptr
            type(c_ptr), intent(in), value :: m
            integer(c_int32_t), intent(in), value :: layer, seq, S, advance
            real(c_float), intent(in) :: x(*)
            real(c_float), intent(inout) :: out(*)
        end function q35_model_layer_forward

        integer(c_int) function q35_model_reset(m) bind(C, name="q35_model_reset")
            import :: c_int, c_ptr
            type(c_ptr), intent(in), value :: m
        end function q35_model_reset

        integer(c_int) function q35_rms_norm(x, weight, output, seq_len, dim) bind(C, name="q35_rms_norm")
            import :: c_int, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: seq_len, dim
            real(c_float), intent(in) :: x(*), weight(*)
            real(c_float), intent(inout) :: output(*)
        end function q35_rms_norm

        integer(c_int) function q35_weights_upload(ctx, format, W_Q, scales, offsets, N, K, src_on_device, out) &
                bind(C, name="q35_weights_upload")
            import :: c_int, c_int8_t, c_int32_t, c_float, c_ptr
            type(c_ptr), intent(in), value :: ctx
            integer(c_int), intent(in), value :: format, src_on_device
            integer(c_int8_t), intent(in) :: W_Q(*)
            real(c_float), intent(in) :: scales(*)
            type(c_ptr), intent(in), value :: offsets
            integer(c_int32_t), intent(in), value :: N, K
            type(c_ptr), intent(out) :: out
        end function q35_weights_upload

        integer(c_int) function q35_weights_free(w) bind(C, name="q35_weights_free")
            import :: c_int, c_ptr
            type(c_ptr), intent(in), value :: w
        end function q35_weights_free

        integer(c_int) function q35_matmul_cached(ctx, w, A, M, C, Out) bind(C, name="q35_matmul_cached")
            import :: c_int, c_int8_t, c_int32_t, c_ptr
            type(c_ptr), intent(in), value :: ctx, w
            integer(c_int8_t), intent(in) :: A(*)
            integer(c_int32_t), intent(in), value :: M
            type(c_ptr), intent(in), value :: C, Out
        end function q35_matmul_cached

        integer(c_int) function q35_matmul_int4_fused(A, W_Q, W_scales, Out, M, N, K) &
                bind(C, name="q35_matmul_int4_fused")
            import :: c_int, c_int8_t, c_int32_t, c_float
            integer(c_int32_t), intent(in), value :: M, N, K
            integer(c_int8_t), intent(in) :: A(*), W_Q(*)
            real(c_float), intent(in) :: W_scales(*)
            real(c_float), intent(inout) :: Out(*)
        end function q35_matmul_int4_fused
    end interface

contains

    ! the shared context, created on first use (device 0, a stream of its own)
    function q35_fortran_context(stat) result(ctx)
        integer, intent(out), optional :: stat
        type(c_ptr) :: ctx
        if (present(stat)) stat = 0
        if (.not. c_associated(fortran_ctx)) then
            call q35_check(q35_ctx_create(0_c_int, c_null_ptr, fortran_ctx), "q35_ctx_create", stat)
        end if
        ctx = fortran_ctx
    end function q35_fortran_context

    subroutine q35_fortran_context_release()
        integer(c_int) :: st
        if (c_associated(fortran_ctx)) then
            st = q35_ctx_destroy(fortran_ctx)
            fortran_ctx = c_null_ptr
        end if
    end subroutine q35_fortran_context_release

end module q35_model_api
