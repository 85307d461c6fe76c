! Drop-in replacement of module llama_model (llama_model.f90) over libq35.so.  Same public
! names; LLaMAModel keeps the reference's components (token_embeddings(vocab, hidden),
! layers(:) of TransformerLayer, final_norm, output_weights(hidden, vocab), num_layers,
! max_seq_len) and gains a device handle.  The first forward_llama uploads the whole model
! from those host arrays to the GPU (one libq35 model: weights repacked once, KV caches,
! the decode kernels) and every later call runs there; like the reference, successive
! calls continue on the KV cache (prefill, then one token at a time).  After editing host
! weights call sync_llama_model (or cleanup_llama_model).  Every procedure takes an
! optional stat=; without it a failure stops with libq35's message (q35_status).
! Compile after transformer_layer.f90.
module llama_model
    use iso_c_binding, only: c_int, c_int32_t, c_ptr, c_null_ptr, c_associated, c_loc
    use iso_fortran_env, only: int32, real32
    use q35_status, only: q35_check
    use q35_model_api
    use transformer_layer
    implicit none
    private
    public :: LLaMAModel, init_llama_model, forward_llama, cleanup_llama_model
    public :: sync_llama_model, model_device_create

    ! llama_model.f90:14-16
    integer(int32), parameter :: NUM_LAYERS = 80
    integer(int32), parameter :: VOCAB_SIZE = 32000
    integer(int32), parameter :: MAX_SEQ_LEN = 2048

    ! llama_model.f90:19-35, plus the device handle
    type :: LLaMAModel
        real(real32), allocatable :: token_embeddings(:,:)
        type(TransformerLayer), allocatable :: layers(:)
        real(real32), allocatable :: final_norm(:)
        real(real32), allocatable :: output_weights(:,:)
        integer(int32) :: num_layers = 0
        integer(int32) :: max_seq_len = 0
        type(c_ptr) :: handle = c_null_ptr
    end type LLaMAModel

contains

    ! llama_model.f90:42-100: the configuration (the reference prints it and allocates
    ! nothing; weights are loaded into the components afterwards)
    subroutine init_llama_model(model)
        type(LLaMAModel), intent(inout) :: model
        print *, "=========================================="
        print *, "Initializing LLaMA 70B Model (libq35, B200)"
        print *, "=========================================="
        print *, "  Layers:", NUM_LAYERS
        print *, "  Hidden dim:", HIDDEN_DIM
        print *, "  Intermediate:", INTERMEDIATE_DIM
        print *, "  Vocab size:", VOCAB_SIZE
        print *, "  Max seq len:", MAX_SEQ_LEN
        model%num_layers = NUM_LAYERS
        model%max_seq_len = MAX_SEQ_LEN
    end subroutine init_llama_model

    ! the device model of a host model of max_batch sequences: configuration from the
    ! arrays, every layer, embeddings, final norm and LM head uploaded
    subroutine model_device_create(layers, token_embeddings, final_norm, output_weights, num_layers, &
                                   max_seq_len, max_batch, handle, stat)
        type(TransformerLayer), intent(in), target :: layers(:)
        real(real32), intent(in), contiguous :: token_embeddings(:,:), final_norm(:), output_weights(:,:)
        integer(int32), intent(in) :: num_layers, max_seq_len, max_batch
        type(c_ptr), intent(out) :: handle
        integer, intent(out), optional :: stat
        type(q35_model_config_t) :: cfg
        type(q35_layer_weights_t) :: lw
        type(c_ptr) :: ctx
        integer :: st, l
        handle = c_null_ptr
        if (present(stat)) stat = 0
        do l = 1, num_layers
            if (.not. layer_weights_loaded(layers(l))) then
                if (present(stat)) then
                    stat = 1
                    return
                end if
                error stop "forward_llama: a layer's weight arrays are not allocated"
            end if
        end do
        ctx = q35_fortran_context(st)
        if (st /= 0) then
            call q35_check(int(st, c_int), "forward_llama", stat)
            return
        end if
        cfg = layer_config(layers(1), num_layers, size(token_embeddings, 1), max_seq_len)
        cfg%max_batch = max_batch
        st = q35_model_create(ctx, cfg, handle)
        do l = 1, num_layers
            if (st /= 0) exit
            lw = layer_weights_view(layers(l))
            st = q35_model_set_layer(handle, int(l - 1, c_int32_t), lw)
        end do
        if (st == 0) st = q35_model_set_embeddings(handle, token_embeddings, final_norm, output_weights)
        if (st /= 0 .and. c_associated(handle)) then
            l = q35_model_destroy(handle)
            handle = c_null_ptr
        end if
        call q35_check(int(st, c_int), "forward_llama (upload)", stat)
    end subroutine model_device_create

    logical function host_model_present(model)
        type(LLaMAModel), intent(in) :: model
        host_model_present = allocated(model%layers) .and. allocated(model%token_embeddings) .and. &
                             allocated(model%final_norm) .and. allocated(model%output_weights)
    end function host_model_present

    ! llama_model.f90:105-147: logits of seq_len tokens (1-based ids) at the model's current
    ! KV-cache position, on the GPU
    subroutine forward_llama(model, token_ids, output_logits, seq_len, stat)
        type(LLaMAModel), intent(inout), target :: model
        integer(int32), intent(in) :: token_ids(:)
        real(real32), intent(out), target, contiguous :: output_logits(:,:)
        integer(int32), intent(in), value :: seq_len
        integer, intent(out), optional :: stat
        integer :: st
        integer(int32) :: l
        if (present(stat)) stat = 0
        if (.not. c_associated(model%handle)) then
            if (.not. host_model_present(model)) then
                if (present(stat)) then
                    stat = 1
                    return
                end if
                error stop "forward_llama: the model's layers, embeddings, final norm or LM head are not allocated"
            end if
            if (model%num_layers <= 0) model%num_layers = size(model%layers)
            if (model%max_seq_len <= 0) model%max_seq_len = MAX_SEQ_LEN
            call model_device_create(model%layers, model%token_embeddings, model%final_norm, model%output_weights, &
                                     model%num_layers, model%max_seq_len, 1, model%handle, st)
            if (st /= 0) then
                call q35_check(int(st, c_int), "forward_llama", stat)
                return
            end if
        end if
        if (size(output_logits, 1) /= seq_len .or. size(token_ids) < seq_len) then
            if (present(stat)) then
                stat = 1
                return
            end if
            error stop "forward_llama: output_logits must be (seq_len, vocab) and token_ids hold seq_len ids"
        end if
        st = q35_model_forward(model%handle, 0_c_int32_t, token_ids, seq_len, c_loc(output_logits))
        if (st == 0) then
            do l = 1, model%num_layers
                model%layers(l)%cache_pos = model%layers(l)%cache_pos + seq_len
            end do
        end if
        call q35_check(int(st, c_int), "forward_llama", stat)
    end subroutine forward_llama

    ! re-upload every layer, the embeddings and the LM head (after editing host weights)
    subroutine sync_llama_model(model, stat)
        type(LLaMAModel), intent(inout), target :: model
        integer, intent(out), optional :: stat
        type(q35_layer_weights_t) :: lw
        integer :: st, l
        if (present(stat)) stat = 0
        if (.not. c_associated(model%handle)) return
        st = 0
        do l = 1, model%num_layers
            if (st /= 0) exit
            lw = layer_weights_view(model%layers(l))
            st = q35_model_set_layer(model%handle, int(l - 1, c_int32_t), lw)
        end do
        if (st == 0) st = q35_model_set_embeddings(model%handle, model%token_embeddings, model%final_norm, &
                                                   model%output_weights)
        call q35_check(int(st, c_int), "sync_llama_model", stat)
    end subroutine sync_llama_model

    ! llama_model.f90:152-179: the device model, then the host arrays
    subroutine cleanup_llama_model(model)
        type(LLaMAModel), intent(inout) :: model
        integer(int32) :: i
        integer(c_int) :: st
        if (c_associated(model%handle)) then
            st = q35_model_destroy(model%handle)
            model%handle = c_null_ptr
        end if
        if (allocated(model%token_embeddings)) deallocate(model%token_embeddings)
        if (allocated(model%final_norm)) deallocate(model%final_norm)
        if (allocated(model%output_weights)) deallocate(model%output_weights)
        if (allocated(model%layers)) then
            do i = 1, size(model%layers)
                call release_layer(model%layers(i))
            end do
            deallocate(model%layers)
        end if
    end subroutine cleanup_llama_model

end module llama_model
