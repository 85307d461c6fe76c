! Drop-in for module weight_loader (weight_loader.f90) over libq35.so.  The reference reads
! one layer's stream-binary file into a TransformerLayer's allocatable arrays; here the
! layer lives in a device model (q35_model_create), so load_layer_weights takes the model
! handle and the 0-based layer index, keeping the file name and the layer number of the
! reference's call (load_layer_weights(layer, filename, layer_idx)).  The 3.5-bit
! safetensors checkpoint (convert_weights_3p5bit.py) loads through load_checkpoint_3p5bit.
! Link: gfortran -c q35_status.f90 weight_loader.f90 && ... -L<pkg> -lq35 -Wl,-rpath,<pkg>
module weight_loader
    use iso_c_binding, only: c_int, c_int32_t, c_char, c_ptr, c_null_char, c_loc
    use q35_status, only: q35_check, q35_error_message
    implicit none
    private
    public :: load_layer_weights, load_checkpoint_3p5bit

    interface
        integer(c_int) function q35_model_load_layer_file(m, layer, path) bind(C, name="q35_model_load_layer_file")
            import :: c_int, c_int32_t, c_char, c_ptr
            type(c_ptr), value :: m
            integer(c_int32_t), value :: layer
            character(kind=c_char), intent(in) :: path(*)
        end function q35_model_load_layer_file
        integer(c_int) function q35_model_load_safetensors(m, paths, n) bind(C, name="q35_model_load_safetensors")
            import :: c_int, c_int32_t, c_ptr
            type(c_ptr), value :: m
            type(c_ptr), intent(in) :: paths(*)
            integer(c_int32_t), value :: n
        end function q35_model_load_safetensors
    end interface

contains

    ! weight_loader.f90:18-182
    subroutine load_layer_weights(model, filename, layer_idx)
        type(c_ptr), intent(in) :: model
        character(len=*), intent(in) :: filename
        integer, intent(in) :: layer_idx
        print '(A,I0,A)', "Loading layer ", layer_idx, " weights..."
        if (q35_model_load_layer_file(model, int(layer_idx, c_int32_t), trim(filename)//c_null_char) /= 0) then
            print *, "  Error loading ", trim(filename), ": ", q35_error_message()
            return
        end if
        print '(A,I0,A)', "  Layer ", layer_idx, " weights loaded successfully"
    end subroutine load_layer_weights

    ! convert_weights_3p5bit.py:105-139 output (model_3p5bit.safetensors)
    subroutine load_checkpoint_3p5bit(model, filename, stat)
        type(c_ptr), intent(in) :: model
        character(len=*), intent(in) :: filename
        integer, intent(out), optional :: stat
        character(kind=c_char, len=:), allocatable, target :: cpath
        type(c_ptr) :: paths(1)
        integer(c_int) :: st
        cpath = trim(filename)//c_null_char
        paths(1) = c_loc(cpath)
        st = q35_model_load_safetensors(model, paths, 1_c_int32_t)
        call q35_check(st, "load_checkpoint_3p5bit", stat)
    end subroutine load_checkpoint_3p5bit

end module weight_loader
